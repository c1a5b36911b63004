"""Kernel-level bindings: call the extern "C" entry points of include/b200ep.h on torch CUDA
tensors (torch provides device memory and the current stream; the arithmetic is the library's).

Each function validates shapes the way the reference's handlers do and raises B200EPError on a
non-zero status.  Nothing here falls back to another implementation.
"""

from __future__ import annotations

import ctypes

from . import check, load_library

DT = {"float32": 1, "float16": 10, "bfloat16": 16}


class GqaParams(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int64), ("seq", ctypes.c_int64), ("num_heads", ctypes.c_int64),
        ("kv_heads", ctypes.c_int64), ("head_size", ctypes.c_int64), ("cap", ctypes.c_int64),
        ("max_seq", ctypes.c_int64), ("rotary_half", ctypes.c_int64), ("do_rotary", ctypes.c_int32),
        ("interleaved", ctypes.c_int32), ("packed_qkv", ctypes.c_int32),
        ("local_window", ctypes.c_int32), ("scale", ctypes.c_float), ("qk_norm_eps", ctypes.c_float),
        ("bias_batch", ctypes.c_int64), ("bias_total", ctypes.c_int64),
    ]


class PagedParams(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int32), ("num_tokens", ctypes.c_int32), ("num_heads", ctypes.c_int32),
        ("kv_heads", ctypes.c_int32), ("head_size", ctypes.c_int32), ("num_blocks", ctypes.c_int32),
        ("block_size", ctypes.c_int32), ("max_blocks", ctypes.c_int32), ("max_seq", ctypes.c_int32),
        ("rotary_half", ctypes.c_int32), ("do_rotary", ctypes.c_int32), ("interleaved", ctypes.c_int32),
        ("scale", ctypes.c_float),
    ]


_configured = False


def _lib():
    global _configured
    L = load_library()
    if not _configured:
        vp, i64, i32, f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
        L.b200ep_matmulnbits.argtypes = [vp, vp, vp, vp, vp, i32, i64, i64, i64, i32, i32, vp]
        L.b200ep_matmulnbits_dequant.argtypes = [vp, vp, vp, vp, i32, i32, i64, i64, i32, i32, vp]
        L.b200ep_rms_norm.argtypes = [vp, vp, vp, i32, i64, i64, f32, vp]
        L.b200ep_skip_rms_norm.argtypes = [vp, vp, vp, vp, vp, i32, i64, i64, f32, vp]
        L.b200ep_gqa_workspace_size.argtypes = [ctypes.POINTER(GqaParams)]
        L.b200ep_gqa_workspace_size.restype = ctypes.c_size_t
        L.b200ep_group_query_attention.argtypes = (
            [ctypes.POINTER(GqaParams)] + [vp] * 12 + [i32, vp, ctypes.c_size_t, vp])
        L.b200ep_matmulnbits_prepack_size.argtypes = [i64, i64, i32, i32, ctypes.POINTER(ctypes.c_size_t)]
        L.b200ep_matmulnbits_prepack.argtypes = [vp, vp, vp, i32, i64, i64, i32, i32, vp, vp]
        L.b200ep_matmulnbits_prepacked.argtypes = [vp, vp, vp, i32, i64, i64, i64, i32, i32, vp]
        L.b200ep_device_error.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int), i32]
        L.b200ep_paged_attention.argtypes = [ctypes.POINTER(PagedParams)] + [vp] * 11 + [i32, vp]
        L.b200ep_gqa_sliding_workspace_size.argtypes = [ctypes.POINTER(GqaParams), i32]
        L.b200ep_gqa_sliding_workspace_size.restype = ctypes.c_size_t
        L.b200ep_group_query_attention_sliding.argtypes = (
            [ctypes.POINTER(GqaParams)] + [vp] * 11 + [i32, vp, ctypes.c_size_t, vp])
        _configured = True
    return L


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device=None):
    import torch

    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _dt(t) -> int:
    return DT[str(t.dtype).replace("torch.", "")]


def device_error(clear: bool = True) -> tuple[int, int]:
    code, detail = ctypes.c_int(0), ctypes.c_int(0)
    check(_lib().b200ep_device_error(ctypes.byref(code), ctypes.byref(detail), int(clear)))
    return code.value, detail.value


def matmulnbits(a, b, scales, zero_points=None, *, K, N, bits=4, block_size=32, out=None):
    """com.microsoft MatMulNBits: a [..., K] -> [..., N] (all float tensors share a dtype)."""
    import torch

    assert a.is_cuda and a.shape[-1] == K and a.is_contiguous()
    M = a.numel() // K
    if out is None:
        out = torch.empty(*a.shape[:-1], N, dtype=a.dtype, device=a.device)
    check(_lib().b200ep_matmulnbits(_p(a), _p(b), _p(scales), _p(zero_points), _p(out), _dt(a), M, N, K,
                                    bits, block_size, _stream(a.device)))
    return out


def matmulnbits_dequant(b, scales, zero_points=None, *, K, N, bits=4, block_size=32, out_dtype=None):
    import torch

    out_dtype = out_dtype or torch.float32
    w = torch.empty(N, K, dtype=out_dtype, device=b.device)
    check(_lib().b200ep_matmulnbits_dequant(_p(b), _p(scales), _p(zero_points), _p(w), _dt(scales),
                                            DT[str(out_dtype).replace("torch.", "")], N, K, bits,
                                            block_size, _stream(b.device)))
    return w


def matmulnbits_prepack(b, scales, zero_points=None, *, K, N, bits=4, block_size=32):
    """Repack ORT-layout int4 weights into tensor-core group records; returns the device buffer."""
    import torch

    size = ctypes.c_size_t(0)
    check(_lib().b200ep_matmulnbits_prepack_size(N, K, bits, block_size, ctypes.byref(size)))
    packed = torch.empty(int(size.value), dtype=torch.uint8, device=b.device)
    check(_lib().b200ep_matmulnbits_prepack(_p(b), _p(scales), _p(zero_points), _dt(scales), N, K, bits, block_size,
                                            _p(packed), _stream(b.device)))
    return packed


def matmulnbits_prepacked(a, packed, *, K, N, bits=4, block_size=32, out=None):
    import torch

    M = a.numel() // K
    if out is None:
        out = torch.empty(*a.shape[:-1], N, dtype=a.dtype, device=a.device)
    check(_lib().b200ep_matmulnbits_prepacked(_p(a), _p(packed), _p(out), _dt(a), M, N, K, bits, block_size,
                                              _stream(a.device)))
    return out


def rms_norm(x, gamma, eps, out=None):
    import torch

    hidden = x.shape[-1]
    out = torch.empty_like(x) if out is None else out
    check(_lib().b200ep_rms_norm(_p(x), _p(gamma), _p(out), _dt(x), x.numel() // hidden, hidden, eps,
                                 _stream(x.device)))
    return out


def skip_rms_norm(x, skip, gamma, eps, *, residual=True):
    import torch

    hidden = x.shape[-1]
    y = torch.empty_like(x)
    r = torch.empty_like(x) if residual else None
    check(_lib().b200ep_skip_rms_norm(_p(x), _p(skip), _p(gamma), _p(y), _p(r), _dt(x), x.numel() // hidden,
                                      hidden, eps, _stream(x.device)))
    return y, r


def gqa_params(*, batch, seq, num_heads, kv_heads, head_size, cap, cos_cache=None, do_rotary=1,
               interleaved=0, packed_qkv=0, local_window=-1, scale=0.0, qk_norm_eps=1e-6,
               attention_bias=None) -> GqaParams:
    p = GqaParams()
    p.batch, p.seq, p.num_heads, p.kv_heads, p.head_size, p.cap = batch, seq, num_heads, kv_heads, head_size, cap
    p.max_seq = 0 if cos_cache is None else cos_cache.shape[0]
    p.rotary_half = 0 if cos_cache is None else cos_cache.shape[1]
    p.do_rotary = int(bool(do_rotary) and cos_cache is not None)
    p.interleaved, p.packed_qkv, p.local_window = int(interleaved), int(packed_qkv), int(local_window)
    p.scale, p.qk_norm_eps = float(scale), float(qk_norm_eps)
    if attention_bias is not None:
        p.bias_batch, p.bias_total = attention_bias.shape[0], attention_bias.shape[-1]
    return p


def group_query_attention(query, key, value, kv_key, kv_value, seqlens_k, cos_cache=None, sin_cache=None,
                          *, num_heads, kv_heads, scale=0.0, do_rotary=1, interleaved=0, local_window=-1,
                          q_norm=None, k_norm=None, qk_norm_eps=1e-6, attention_bias=None, out=None,
                          workspace=None):
    """GroupQueryAttention over the shared KV buffers kv_key/kv_value [B, HK, cap, D] (in place)."""
    import torch

    packed = key is None
    B, S, W = query.shape
    D = W // (num_heads + 2 * kv_heads) if packed else W // num_heads
    p = gqa_params(batch=B, seq=S, num_heads=num_heads, kv_heads=kv_heads, head_size=D, cap=kv_key.shape[2],
                   cos_cache=cos_cache, do_rotary=do_rotary, interleaved=interleaved, packed_qkv=packed,
                   local_window=local_window, scale=scale, qk_norm_eps=qk_norm_eps,
                   attention_bias=attention_bias)
    if out is None:
        out = torch.empty(B, S, num_heads * D, dtype=query.dtype, device=query.device)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    check(_lib().b200ep_group_query_attention(
        ctypes.byref(p), _p(query), _p(key), _p(value), _p(kv_key), _p(kv_value), _p(seqlens_k),
        _p(cos_cache), _p(sin_cache), _p(q_norm), _p(k_norm), _p(attention_bias), _p(out), _dt(query),
        _p(workspace), ws_bytes, _stream(query.device)))
    return out


def group_query_attention_sliding(query, key, value, past_key, past_value, seqlens_k, cos_cache=None,
                                  sin_cache=None, *, num_heads, kv_heads, local_window, scale=0.0, do_rotary=1,
                                  interleaved=0, present_key=None, present_value=None, out=None):
    """GroupQueryAttention with sliding_window_cache = 1: returns (out, present_key, present_value);
    present defaults to the past buffers (updated in place)."""
    import torch

    packed = key is None
    B, S, W = query.shape
    D = W // (num_heads + 2 * kv_heads) if packed else W // num_heads
    p = gqa_params(batch=B, seq=S, num_heads=num_heads, kv_heads=kv_heads, head_size=D, cap=past_key.shape[2],
                   cos_cache=cos_cache, do_rotary=do_rotary, interleaved=interleaved, packed_qkv=packed,
                   local_window=local_window, scale=scale)
    present_key = past_key if present_key is None else present_key
    present_value = past_value if present_value is None else present_value
    if out is None:
        out = torch.empty(B, S, num_heads * D, dtype=query.dtype, device=query.device)
    check(_lib().b200ep_group_query_attention_sliding(
        ctypes.byref(p), _p(query), _p(key), _p(value), _p(past_key), _p(past_value), _p(present_key),
        _p(present_value), _p(seqlens_k), _p(cos_cache), _p(sin_cache), _p(out), _dt(query), None, 0,
        _stream(query.device)))
    return out, present_key, present_value


def gqa_workspace_size(**kw) -> int:
    return int(_lib().b200ep_gqa_workspace_size(ctypes.byref(gqa_params(**kw))))


def paged_attention(query, key, value, key_cache, value_cache, cumulative_seqlens, past_seqlens, block_table,
                    cos_cache=None, sin_cache=None, *, num_heads, kv_heads, scale=0.0, interleaved=0, out=None):
    """com.microsoft PagedAttention: packed rows [num_tokens, H*D]; caches [num_blocks, block_size, HK, D]
    updated in place; control tensors int32 on the device."""
    import torch

    T, W = query.shape
    D = W // num_heads
    batch = cumulative_seqlens.numel() - 1
    p = PagedParams()
    p.batch, p.num_tokens, p.num_heads, p.kv_heads, p.head_size = batch, T, num_heads, kv_heads, D
    p.num_blocks, p.block_size = key_cache.shape[0], key_cache.shape[1]
    p.max_blocks = block_table.numel() // batch
    p.do_rotary = int(cos_cache is not None)
    p.max_seq = 0 if cos_cache is None else cos_cache.shape[0]
    p.rotary_half = 0 if cos_cache is None else cos_cache.shape[1]
    p.interleaved, p.scale = int(interleaved), float(scale)
    if out is None:
        out = torch.empty(T, num_heads * D, dtype=query.dtype, device=query.device)
    check(_lib().b200ep_paged_attention(
        ctypes.byref(p), _p(query), _p(key), _p(value), _p(key_cache), _p(value_cache), _p(cumulative_seqlens),
        _p(past_seqlens), _p(block_table), _p(cos_cache), _p(sin_cache), _p(out), _dt(query),
        _stream(query.device)))
    return out
