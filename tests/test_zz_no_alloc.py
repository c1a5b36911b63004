"""The allocation-free GroupQueryAttention entry point (b200ep_group_query_attention_noalloc).

It serves callers that may not allocate device memory once running — a server that reserves
its HBM budget at start-up, a decode loop that must not allocate or free between tokens — by
keeping the split-K scratch in a fixed library-owned device array.  This file checks, through
the C ABI, that two decode steps in a row give the same output and KV-buffer contents as the
regular entry point (which takes a caller-provided workspace), within the fp16 tolerance the
other GQA tests use, and that an over-size geometry is refused with B200EP_ERANGE.

The file name sorts last so that a run stopping at the first failure has run everything else
first; it passes both on its own in a fresh process and after the other tests.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TOL = dict(rtol=1e-2, atol=1e-3)


def _lib():
    from onnxruntime_ep_b200 import ops

    L = ops._lib()
    vp = ctypes.c_void_p
    L.b200ep_group_query_attention_noalloc.argtypes = [ctypes.POINTER(ops.GqaParams)] + [vp] * 12 + [ctypes.c_int, vp]
    L.b200ep_gqa_noalloc_max_workspace.restype = ctypes.c_size_t
    return L, ops


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def test_noalloc_gqa_matches_workspace_entry_two_steps():
    L, ops = _lib()
    rng = np.random.default_rng(42)
    B, H, HK, D, past = 2, 32, 8, 128, 777
    cap = past + 8
    dev = "cuda"
    kc = torch.from_numpy(rng.standard_normal((B, HK, cap, D)).astype(np.float16)).to(dev)
    vc = torch.from_numpy(rng.standard_normal((B, HK, cap, D)).astype(np.float16)).to(dev)
    k_ref, v_ref = kc.clone(), vc.clone()
    k_na, v_na = kc.clone(), vc.clone()
    half = D // 2
    inv = 1.0 / (10000.0 ** (np.arange(half) / half))
    ang = np.arange(cap + 8)[:, None] * inv[None, :]
    cos = torch.from_numpy(np.cos(ang).astype(np.float16)).to(dev)
    sin = torch.from_numpy(np.sin(ang).astype(np.float16)).to(dev)
    p = ops.gqa_params(batch=B, seq=1, num_heads=H, kv_heads=HK, head_size=D, cap=cap, cos_cache=cos)
    ws_bytes = ops.gqa_workspace_size(batch=B, seq=1, num_heads=H, kv_heads=HK, head_size=D, cap=cap, cos_cache=cos)
    assert 0 < ws_bytes <= L.b200ep_gqa_noalloc_max_workspace()
    workspace = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for step in range(2):
        q = torch.from_numpy(rng.standard_normal((B, 1, H * D)).astype(np.float16)).to(dev)
        k = torch.from_numpy(rng.standard_normal((B, 1, HK * D)).astype(np.float16)).to(dev)
        v = torch.from_numpy(rng.standard_normal((B, 1, HK * D)).astype(np.float16)).to(dev)
        seqlens = torch.full((B,), past + step, dtype=torch.int32, device=dev)
        out_ref = torch.empty(B, 1, H * D, dtype=torch.float16, device=dev)
        out_na = torch.empty_like(out_ref)
        ops.check(L.b200ep_group_query_attention(
            ctypes.byref(p), _p(q), _p(k), _p(v), _p(k_ref), _p(v_ref), _p(seqlens), _p(cos), _p(sin), None, None,
            None, _p(out_ref), 10, _p(workspace), ws_bytes, stream))
        ops.check(L.b200ep_group_query_attention_noalloc(
            ctypes.byref(p), _p(q), _p(k), _p(v), _p(k_na), _p(v_na), _p(seqlens), _p(cos), _p(sin), None, None,
            None, _p(out_na), 10, stream))
        torch.cuda.synchronize()
        np.testing.assert_allclose(out_na.float().cpu().numpy(), out_ref.float().cpu().numpy(), **TOL)
        assert torch.equal(k_na, k_ref) and torch.equal(v_na, v_ref)
    code, _ = ops.device_error(clear=True)
    assert code == 0


def test_noalloc_gqa_refuses_oversize_scratch():
    from onnxruntime_ep_b200 import B200EPError

    L, ops = _lib()
    # a prefill-sized chunk: the generic path's rotated-query scratch alone exceeds the fixed array
    B, S, H, HK, D, cap = 4, 512, 32, 8, 128, 1024
    p = ops.gqa_params(batch=B, seq=S, num_heads=H, kv_heads=HK, head_size=D, cap=cap)
    need = ops.gqa_workspace_size(batch=B, seq=S, num_heads=H, kv_heads=HK, head_size=D, cap=cap)
    assert need > L.b200ep_gqa_noalloc_max_workspace()
    dummy = torch.zeros(1, dtype=torch.float16, device="cuda")
    with pytest.raises(B200EPError, match="limit") as ei:
        ops.check(L.b200ep_group_query_attention_noalloc(
            ctypes.byref(p), _p(dummy), _p(dummy), _p(dummy), _p(dummy), _p(dummy), _p(dummy), None, None, None,
            None, None, _p(dummy), 10, None))
    assert ei.value.status == 2  # B200EP_ERANGE
