"""ctypes wrapper over the CPU oracle (liboracle.so) — TEST INFRASTRUCTURE ONLY.

Only tests, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py``
may import this module.  The product library never calls it.

Every function mirrors one operator of the reference's hot path with ORT CPU
semantics (see oracle.c for the file:line each one restates) and takes/returns
numpy arrays.  fp16 arrays are numpy float16; bf16 arrays are passed as uint16
bit patterns together with ``dtype="bf16"``.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

DT_F32, DT_U8, DT_I32, DT_F16, DT_BF16 = 1, 2, 6, 10, 16
_DT_CODES = {"f32": DT_F32, "f16": DT_F16, "bf16": DT_BF16}


class OracleError(RuntimeError):
    pass


class GqaParams(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int64),
        ("seq", ctypes.c_int64),
        ("num_heads", ctypes.c_int64),
        ("kv_heads", ctypes.c_int64),
        ("head_size", ctypes.c_int64),
        ("past_cap", ctypes.c_int64),
        ("present_cap", ctypes.c_int64),
        ("max_seq", ctypes.c_int64),
        ("rotary_half", ctypes.c_int64),
        ("do_rotary", ctypes.c_int32),
        ("interleaved", ctypes.c_int32),
        ("packed_qkv", ctypes.c_int32),
        ("shared_buffer", ctypes.c_int32),
        ("local_window", ctypes.c_int32),
        ("has_qk_norm", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("qk_norm_eps", ctypes.c_float),
        ("bias_batch", ctypes.c_int64),
        ("bias_total", ctypes.c_int64),
    ]


_lib = None


def build() -> str:
    """Compile liboracle.so with the committed Makefile (no-op when up to date)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        vp, i64, i32, f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
        L.oracle_matmulnbits_dequant.argtypes = [vp, vp, i32, vp, i64, i64, i32, i32, vp]
        L.oracle_matmulnbits.argtypes = [vp, vp, vp, vp, vp, i32, i64, i64, i64, i32, i32, i32]
        L.oracle_rms_norm.argtypes = [vp, vp, vp, i32, i64, i64, f32, i32]
        L.oracle_skip_rms_norm.argtypes = [vp, vp, vp, vp, vp, i32, i64, i64, f32, i32]
        L.oracle_gqa.argtypes = [ctypes.POINTER(GqaParams)] + [vp] * 14 + [i32, i32]
        L.oracle_gqa_sliding.argtypes = [ctypes.POINTER(GqaParams)] + [vp] * 11 + [i32, i32]
        L.oracle_gather_block_quantized.argtypes = [vp, vp, i32, vp, vp, i64, i64, i64, i32, vp, i32]
        L.oracle_half_to_float.argtypes = [ctypes.c_uint16]
        L.oracle_half_to_float.restype = ctypes.c_float
        L.oracle_float_to_half.argtypes = [ctypes.c_float]
        L.oracle_float_to_half.restype = ctypes.c_uint16
        L.oracle_float_to_bf16.argtypes = [ctypes.c_float]
        L.oracle_float_to_bf16.restype = ctypes.c_uint16
        L.oracle_bf16_to_float.argtypes = [ctypes.c_uint16]
        L.oracle_bf16_to_float.restype = ctypes.c_float
        L.oracle_max_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _dtype_code(a: np.ndarray, dtype: str | None) -> int:
    if dtype is not None:
        return _DT_CODES[dtype]
    if a.dtype == np.float32:
        return DT_F32
    if a.dtype == np.float16:
        return DT_F16
    raise OracleError(f"unsupported float dtype {a.dtype}; pass dtype='bf16' for uint16 bf16 bits")


def _np_dtype(code: int):
    return {DT_F32: np.float32, DT_F16: np.float16, DT_BF16: np.uint16}[code]


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise OracleError(f"{what} failed with status {rc}")


def max_threads() -> int:
    return int(lib().oracle_max_threads())


# ---- conversions (the oracle's RNE implementations, exposed for self-tests) ------------------
def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns, round-to-nearest-even (vectorised restatement of oracle.c)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---- MatMulNBits --------------------------------------------------------------------------------
def matmulnbits_dequant(b, scales, zero_points, *, N, K, bits=4, block_size=32, dtype=None):
    """Dequantised weight W[N, K] as fp32: (q - zp) * scale (bit-exact target)."""
    b = np.ascontiguousarray(b, dtype=np.uint8)
    scales = np.ascontiguousarray(scales)
    zp = None if zero_points is None else np.ascontiguousarray(zero_points, dtype=np.uint8)
    w = np.empty((N, K), dtype=np.float32)
    rc = lib().oracle_matmulnbits_dequant(_ptr(b), _ptr(scales), _dtype_code(scales, dtype), _ptr(zp),
                                          N, K, bits, block_size, _ptr(w))
    _check(rc, "oracle_matmulnbits_dequant")
    return w


def matmulnbits(a, b, scales, zero_points=None, *, N, K, bits=4, block_size=32, dtype=None,
                threads=0):
    """Y[..., N] = A[..., K] . dequant(B)^T with ORT CPU semantics (quant.rs:986-1130)."""
    a = np.ascontiguousarray(a)
    code = _dtype_code(a, dtype)
    b = np.ascontiguousarray(b, dtype=np.uint8)
    scales = np.ascontiguousarray(scales)
    zp = None if zero_points is None else np.ascontiguousarray(zero_points, dtype=np.uint8)
    M = int(np.prod(a.shape[:-1])) if a.ndim > 1 else 1
    y = np.empty(tuple(a.shape[:-1]) + (N,), dtype=_np_dtype(code))
    rc = lib().oracle_matmulnbits(_ptr(a), _ptr(b), _ptr(scales), _ptr(zp), _ptr(y), code, M, N, K,
                                  bits, block_size, threads)
    _check(rc, "oracle_matmulnbits")
    return y


# ---- norms --------------------------------------------------------------------------------------
def rms_norm(x, gamma, eps, *, dtype=None, threads=0):
    x = np.ascontiguousarray(x)
    gamma = np.ascontiguousarray(gamma)
    code = _dtype_code(x, dtype)
    hidden = x.shape[-1]
    rows = x.size // hidden
    y = np.empty_like(x)
    _check(lib().oracle_rms_norm(_ptr(x), _ptr(gamma), _ptr(y), code, rows, hidden, eps, threads),
           "oracle_rms_norm")
    return y


def skip_rms_norm(x, skip, gamma, eps, *, dtype=None, threads=0):
    """Returns (normalised, residual_sum)."""
    x = np.ascontiguousarray(x)
    skip = np.ascontiguousarray(skip)
    gamma = np.ascontiguousarray(gamma)
    code = _dtype_code(x, dtype)
    hidden = x.shape[-1]
    rows = x.size // hidden
    y = np.empty_like(x)
    r = np.empty_like(x)
    _check(lib().oracle_skip_rms_norm(_ptr(x), _ptr(skip), _ptr(gamma), _ptr(y), _ptr(r), code, rows,
                                      hidden, eps, threads), "oracle_skip_rms_norm")
    return y, r


# ---- GroupQueryAttention ------------------------------------------------------------------------
def gqa(query, key, value, past_key, past_value, seqlens_k, cos_cache=None, sin_cache=None, *,
        num_heads, kv_heads, scale=0.0, do_rotary=1, interleaved=0, present_cap=None,
        shared_buffer=False, local_window=-1, q_norm=None, k_norm=None, qk_norm_eps=1e-6,
        attention_bias=None, dtype=None, threads=0):
    """GroupQueryAttention with ORT CPU semantics (attention.rs:556-952).

    ``key``/``value`` None means packed QKV in ``query``.  Returns
    (attn_output [B,S,H*D], present_key, present_value).  With ``shared_buffer``
    the past arrays are updated in place and returned as present.
    """
    query = np.ascontiguousarray(query)
    code = _dtype_code(query, dtype)
    packed = key is None
    B, S, width = query.shape
    D = width // (num_heads + 2 * kv_heads) if packed else width // num_heads
    past_cap = 0 if past_key is None else past_key.shape[2]
    if present_cap is None:
        present_cap = past_cap if shared_buffer else past_cap + S
    p = GqaParams()
    p.batch, p.seq, p.num_heads, p.kv_heads, p.head_size = B, S, num_heads, kv_heads, D
    p.past_cap, p.present_cap = past_cap, present_cap
    p.max_seq = 0 if cos_cache is None else cos_cache.shape[0]
    p.rotary_half = 0 if cos_cache is None else cos_cache.shape[1]
    p.do_rotary, p.interleaved, p.packed_qkv = int(do_rotary), int(interleaved), int(packed)
    p.shared_buffer = int(shared_buffer)
    p.local_window = int(local_window)
    p.has_qk_norm = int(q_norm is not None)
    p.scale, p.qk_norm_eps = float(scale), float(qk_norm_eps)
    if attention_bias is not None:
        p.bias_batch, p.bias_total = attention_bias.shape[0], attention_bias.shape[-1]
    npdt = _np_dtype(code)
    if shared_buffer:
        pk, pv = past_key, past_value
        assert pk.flags.c_contiguous and pv.flags.c_contiguous
    else:
        pk = np.empty((B, kv_heads, present_cap, D), dtype=npdt)
        pv = np.empty_like(pk)
    out = np.empty((B, S, num_heads * D), dtype=npdt)
    seqlens = np.ascontiguousarray(seqlens_k, dtype=np.int32)
    args = [
        query, None if packed else np.ascontiguousarray(key),
        None if packed else np.ascontiguousarray(value),
        None if past_key is None else np.ascontiguousarray(past_key),
        None if past_value is None else np.ascontiguousarray(past_value), seqlens,
        None if cos_cache is None else np.ascontiguousarray(cos_cache),
        None if sin_cache is None else np.ascontiguousarray(sin_cache),
        None if q_norm is None else np.ascontiguousarray(q_norm),
        None if k_norm is None else np.ascontiguousarray(k_norm),
        None if attention_bias is None else np.ascontiguousarray(attention_bias), out, pk, pv,
    ]
    rc = lib().oracle_gqa(ctypes.byref(p), *[_ptr(x) for x in args], code, threads)
    _check(rc, "oracle_gqa")
    return out, pk, pv


def gqa_sliding(query, key, value, past_key, past_value, seqlens_k, cos_cache=None, sin_cache=None, *,
                num_heads, kv_heads, local_window, scale=0.0, do_rotary=1, interleaved=0, dtype=None, threads=0):
    """GroupQueryAttention with sliding_window_cache = 1 (attention.rs:725-880): past_key /
    past_value [B, kv_heads, cap, D] hold the resident rows; returns (attn_output, present_key,
    present_value) with present at the same capacity (rows beyond the resident ones zero)."""
    query = np.ascontiguousarray(query)
    code = _dtype_code(query, dtype)
    B, S, width = query.shape
    D = width // num_heads
    cap = past_key.shape[2]
    p = GqaParams()
    p.batch, p.seq, p.num_heads, p.kv_heads, p.head_size = B, S, num_heads, kv_heads, D
    p.past_cap = p.present_cap = cap
    p.max_seq = 0 if cos_cache is None else cos_cache.shape[0]
    p.rotary_half = 0 if cos_cache is None else cos_cache.shape[1]
    p.do_rotary, p.interleaved = int(do_rotary), int(interleaved)
    p.shared_buffer, p.local_window, p.scale = 1, int(local_window), float(scale)
    npdt = _np_dtype(code)
    out = np.empty((B, S, num_heads * D), dtype=npdt)
    pk = np.empty((B, kv_heads, cap, D), dtype=npdt)
    pv = np.empty_like(pk)
    args = [query, np.ascontiguousarray(key), np.ascontiguousarray(value), np.ascontiguousarray(past_key),
            np.ascontiguousarray(past_value), np.ascontiguousarray(seqlens_k, dtype=np.int32),
            None if cos_cache is None else np.ascontiguousarray(cos_cache),
            None if sin_cache is None else np.ascontiguousarray(sin_cache), out, pk, pv]
    rc = lib().oracle_gqa_sliding(ctypes.byref(p), *[_ptr(x) for x in args], code, threads)
    _check(rc, "oracle_gqa_sliding")
    return out, pk, pv


class PagedParams(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int64),
        ("num_tokens", ctypes.c_int64),
        ("num_heads", ctypes.c_int64),
        ("kv_heads", ctypes.c_int64),
        ("head_size", ctypes.c_int64),
        ("num_blocks", ctypes.c_int64),
        ("block_size", ctypes.c_int64),
        ("max_blocks", ctypes.c_int64),
        ("max_seq", ctypes.c_int64),
        ("rotary_half", ctypes.c_int64),
        ("do_rotary", ctypes.c_int32),
        ("interleaved", ctypes.c_int32),
        ("scale", ctypes.c_float),
    ]


def paged_attention(query, key, value, key_cache, value_cache, cum_seqlens, past_seqlens, block_table,
                    cos_cache=None, sin_cache=None, *, num_heads, kv_heads, scale=0.0, interleaved=0,
                    dtype=None, threads=0):
    """PagedAttention with the reference's semantics (attention.rs:2495-2746).

    Returns (output [num_tokens, H*D], key_cache, value_cache); the caches are copies with the
    new rows scattered in.
    """
    query = np.ascontiguousarray(query)
    code = _dtype_code(query, dtype)
    T, width = query.shape
    D = width // num_heads
    kc, vc = np.array(key_cache, copy=True, order="C"), np.array(value_cache, copy=True, order="C")
    cum = np.ascontiguousarray(cum_seqlens, dtype=np.int32)
    past = np.ascontiguousarray(past_seqlens, dtype=np.int32)
    bt = np.ascontiguousarray(block_table, dtype=np.int32)
    p = PagedParams()
    p.batch, p.num_tokens, p.num_heads, p.kv_heads, p.head_size = len(cum) - 1, T, num_heads, kv_heads, D
    p.num_blocks, p.block_size, p.max_blocks = kc.shape[0], kc.shape[1], bt.size // (len(cum) - 1)
    p.do_rotary = int(cos_cache is not None)
    p.max_seq = 0 if cos_cache is None else cos_cache.shape[0]
    p.rotary_half = 0 if cos_cache is None else cos_cache.shape[1]
    p.interleaved, p.scale = int(interleaved), float(scale)
    out = np.empty((T, num_heads * D), dtype=_np_dtype(code))
    args = [query, np.ascontiguousarray(key), np.ascontiguousarray(value), kc, vc, cum, past, bt,
            None if cos_cache is None else np.ascontiguousarray(cos_cache),
            None if sin_cache is None else np.ascontiguousarray(sin_cache), out]
    rc = lib().oracle_paged_attention(ctypes.byref(p), *[_ptr(x) for x in args], code, threads)
    _check(rc, "oracle_paged_attention")
    return out, kc, vc


def gather_block_quantized(data, scales, indices, *, block_size, zero_points=None, dtype=None):
    data = np.ascontiguousarray(data, dtype=np.uint8)
    scales = np.ascontiguousarray(scales)
    idx = np.ascontiguousarray(indices, dtype=np.int64)
    vocab, dim = data.shape[0], data.shape[1] * 2
    code = _dtype_code(scales, dtype)
    out = np.empty(tuple(idx.shape) + (dim,), dtype=_np_dtype(code))
    zp = None if zero_points is None else np.ascontiguousarray(zero_points, dtype=np.uint8)
    rc = lib().oracle_gather_block_quantized(_ptr(data), _ptr(scales), code, _ptr(zp), _ptr(idx),
                                             idx.size, vocab, dim, block_size, _ptr(out), code)
    _check(rc, "oracle_gather_block_quantized")
    return out
