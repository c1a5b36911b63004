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


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_noalloc_gqa_prompt_matches_oracle(dt):
    """A prompt (S = 64 after 100 cached rows, 32 / 8 heads of 128) whose workspace fits the fixed
    scratch: the no-alloc entry against the oracle of the GroupQueryAttention semantics, the KV
    append bit-exact."""
    from oracle import oracle

    L, ops = _lib()
    rng = np.random.default_rng(7 if dt == "f16" else 8)
    B, S, H, HK, D, past = 1, 64, 32, 8, 128, 100
    cap = past + S + 4
    q = rng.standard_normal((B, S, H * D)).astype(np.float32)
    k = rng.standard_normal((B, S, HK * D)).astype(np.float32)
    v = rng.standard_normal((B, S, HK * D)).astype(np.float32)
    kc = np.zeros((B, HK, cap, D), np.float32)
    vc = np.zeros((B, HK, cap, D), np.float32)
    kc[:, :, :past] = rng.standard_normal((B, HK, past, D))
    vc[:, :, :past] = rng.standard_normal((B, HK, past, D))
    half = D // 2
    ang = np.arange(cap + 8)[:, None] * (1.0 / (10000.0 ** (np.arange(half) / half)))[None, :]
    cos, sin = np.cos(ang), np.sin(ang)
    seqlens = np.full((B,), past + S - 1, np.int32)
    if dt == "f16":
        args = [x.astype(np.float16) for x in (q, k, v, kc, vc, cos, sin)]
        dev = [torch.from_numpy(x).cuda() for x in args]
        code, tol = 10, TOL
    else:
        args = [oracle.f32_to_bf16_bits(x.astype(np.float32)) for x in (q, k, v, kc, vc, cos, sin)]
        dev = [torch.from_numpy(x).cuda().view(torch.bfloat16) for x in args]
        code, tol = 16, TOL
    want, wk, wv = oracle.gqa(args[0], args[1], args[2], args[3].copy(), args[4].copy(), seqlens, args[5], args[6],
                              num_heads=H, kv_heads=HK, shared_buffer=True, dtype="bf16" if dt == "bf16" else None)
    p = ops.gqa_params(batch=B, seq=S, num_heads=H, kv_heads=HK, head_size=D, cap=cap, cos_cache=dev[5])
    out = torch.empty(B, S, H * D, dtype=dev[0].dtype, device="cuda")
    sl = torch.from_numpy(seqlens).cuda()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    ops.check(L.b200ep_group_query_attention_noalloc(
        ctypes.byref(p), _p(dev[0]), _p(dev[1]), _p(dev[2]), _p(dev[3]), _p(dev[4]), _p(sl), _p(dev[5]), _p(dev[6]),
        None, None, None, _p(out), code, stream))
    torch.cuda.synchronize()
    if dt == "f16":
        got = out.float().cpu().numpy()
        np.testing.assert_allclose(got, want.astype(np.float32), **tol)
        np.testing.assert_array_equal(dev[3].cpu().numpy(), wk)
        np.testing.assert_array_equal(dev[4].cpu().numpy(), wv)
    else:
        got = out.float().cpu().numpy()
        np.testing.assert_allclose(got, oracle.bf16_bits_to_f32(want), **tol)
        np.testing.assert_array_equal(dev[3].view(torch.int16).cpu().numpy().view(np.uint16), wk)
    code_e, _ = ops.device_error(clear=True)
    assert code_e == 0
