"""TEST INFRASTRUCTURE ONLY: ctypes wrapper of the CPU oracle (mc_oracle.c).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may use
this package, as the checker or the timed CPU baseline; the product never
does. Parity is unpinned by the reference's own tests (it has none and cannot
run here); see the header of mc_oracle.c.

All arrays are numpy arrays: bf16 as uint16 bit patterns, u32 as uint32.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import build as _build

_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        exact, _ = _build.build()
        _lib = C.CDLL(str(exact))
        _lib.or_exp.restype = C.c_float
        _lib.or_exp.argtypes = [C.c_float]
        _lib.or_silu.restype = C.c_float
        _lib.or_silu.argtypes = [C.c_float]
        _lib.or_sigmoid.restype = C.c_float
        _lib.or_sigmoid.argtypes = [C.c_float]
        _lib.or_f32_to_bf16.restype = C.c_uint16
        _lib.or_f32_to_bf16.argtypes = [C.c_float]
        _lib.or_argmax_key.restype = C.c_uint64
        _lib.or_argmax_key.argtypes = [C.c_float, C.c_uint32]
    return _lib


def _ptr(a):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be contiguous"
    return a.ctypes.data_as(C.c_void_p)


def exp(x: float) -> float:
    return lib().or_exp(x)


def silu(x: float) -> float:
    return lib().or_silu(x)


def sigmoid(x: float) -> float:
    return lib().or_sigmoid(x)


def f32_to_bf16(x: float) -> int:
    return lib().or_f32_to_bf16(x)


def argmax_key(v: float, i: int) -> int:
    return lib().or_argmax_key(v, i)


def gemv_quant(codes, scales, biases, bits, x, with_acc=False):
    """y bf16 [B, N] (and fp32 sums) for codes [N, K*bits/32], x bf16 [B, K]."""
    n = codes.shape[0]
    k = codes.shape[1] * 32 // bits
    x = np.ascontiguousarray(x.reshape(-1, k))
    b = x.shape[0]
    y = np.zeros((b, n), np.uint16)
    acc = np.zeros((b, n), np.float32) if with_acc else None
    lib().or_gemv_quant(_ptr(codes), _ptr(scales), _ptr(biases), bits, n, k, _ptr(x), b,
                        _ptr(y), _ptr(acc))
    return (y, acc) if with_acc else y


def head_argmax(codes, scales, biases, bits, x):
    n = codes.shape[0]
    k = codes.shape[1] * 32 // bits
    x = np.ascontiguousarray(x.reshape(-1, k))
    b = x.shape[0]
    keys = np.zeros(b, np.uint64)
    toks = np.zeros(b, np.uint32)
    lib().or_head_argmax(_ptr(codes), _ptr(scales), _ptr(biases), bits, n, k, _ptr(x), b,
                         _ptr(keys), _ptr(toks))
    return keys, toks


def argmax_bf16(logits):
    logits = np.ascontiguousarray(logits)
    n = logits.shape[-1]
    b = logits.size // n
    out = np.zeros(b, np.uint32)
    lib().or_argmax_bf16(_ptr(logits), n, b, _ptr(out))
    return out


def add_rmsnorm(h, b, w, eps=1e-5):
    h = np.ascontiguousarray(h)
    hout = np.zeros_like(h)
    nout = np.zeros_like(h)
    H = h.shape[-1]
    rows = h.size // H
    for r in range(rows):
        lib().or_add_rmsnorm(_ptr(h.reshape(rows, H)[r]),
                             None if b is None else _ptr(np.ascontiguousarray(b.reshape(rows, H)[r])),
                             _ptr(w), H, C.c_float(eps), _ptr(hout.reshape(rows, H)[r]),
                             _ptr(nout.reshape(rows, H)[r]))
    return hout, nout


def router_logits(normed, w, w_dtype):
    e, k = w.shape
    normed = np.ascontiguousarray(normed)
    rows = normed.size // k
    out = np.zeros((rows, e), np.float32)
    for r in range(rows):
        lib().or_router_logits(_ptr(np.ascontiguousarray(normed.reshape(rows, k)[r])), _ptr(w),
                               w_dtype, e, k, _ptr(out[r]))
    return out


def route_topk(z, mode, bias=None, eps=1e-6):
    z = np.ascontiguousarray(z, dtype=np.float32)
    e = z.shape[-1]
    rows = z.size // e
    ids = np.zeros((rows, 4), np.uint32)
    w = np.zeros((rows, 4), np.uint16)
    for r in range(rows):
        lib().or_route_topk(_ptr(z.reshape(rows, e)[r]), e, 4, mode, _ptr(bias), C.c_float(eps),
                            _ptr(ids[r]), _ptr(w[r]))
    return ids, w


def router_addnorm_route(h, b, norm_w, w, w_dtype, ebias, mode, eps=1e-5, route_eps=1e-6):
    """Returns (hout, normed, logits, ids, weights) for rows of h [B, 2048]."""
    e, H = w.shape
    h = np.ascontiguousarray(h.reshape(-1, H))
    B = h.shape[0]
    b = None if b is None else np.ascontiguousarray(b.reshape(B, H))
    hout = np.zeros_like(h)
    normed = np.zeros_like(h)
    logits = np.zeros((B, e), np.float32)
    ids = np.zeros((B, 4), np.uint32)
    wts = np.zeros((B, 4), np.uint16)
    lib().or_router_addnorm_route(_ptr(h), _ptr(b), _ptr(norm_w), _ptr(w), w_dtype, _ptr(ebias),
                                  mode, e, H, C.c_float(eps), C.c_float(route_eps), B,
                                  _ptr(hout), _ptr(normed), _ptr(logits), _ptr(ids), _ptr(wts))
    return hout, normed, logits, ids, wts


def gemv_gather_act(gate, up, x, ids, n_experts=64):
    """gate/up: (codes, scales, biases) stacked [E*I, H]; x [B, H]; ids [B, 4]."""
    gc, gs, gb = gate
    uc, us, ub = up
    H = gc.shape[1] * 8
    x = np.ascontiguousarray(x.reshape(-1, H))
    B = x.shape[0]
    ids = np.ascontiguousarray(ids.reshape(B, 4), dtype=np.uint32)
    I = gc.shape[0] // n_experts
    act = np.zeros((B, 4, I), np.uint16)
    lib().or_gemv_gather_act(_ptr(gc), _ptr(gs), _ptr(gb), _ptr(uc), _ptr(us), _ptr(ub), I, H,
                             _ptr(x), _ptr(ids), B, _ptr(act))
    return act


def gemv_gather_down_combine4(down, act, ids, wts, n_experts=64):
    dc, ds, db = down
    I = dc.shape[1] * 8
    H = dc.shape[0] // n_experts
    B = ids.size // 4
    act = np.ascontiguousarray(act.reshape(B, 4, I))
    out = np.zeros((B, H), np.uint16)
    lib().or_gemv_gather_down_combine4(_ptr(dc), _ptr(ds), _ptr(db), H, I, _ptr(act),
                                       _ptr(np.ascontiguousarray(ids, dtype=np.uint32)),
                                       _ptr(np.ascontiguousarray(wts)), B, _ptr(out))
    return out


def moe_route_batch(logits, mode=0, bias=None, eps=1e-6):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    m, e = logits.shape
    ids = np.zeros((m, 4), np.uint32)
    gw = np.zeros((m, 4), np.uint16)
    lib().or_moe_route_batch(_ptr(logits), m, e, mode, _ptr(bias), C.c_float(eps), _ptr(ids),
                             _ptr(gw))
    return ids, gw


def moe_sort(ids, n_experts=64):
    ids = np.ascontiguousarray(ids, dtype=np.uint32)
    m = ids.shape[0]
    counts = np.zeros(n_experts, np.uint32)
    offsets = np.zeros(n_experts, np.uint32)
    ids_sorted = np.zeros(m * 4, np.uint32)
    slotpos = np.zeros(m * 4, np.uint32)
    lib().or_moe_sort(_ptr(ids), m, 4, n_experts, _ptr(counts), _ptr(offsets), _ptr(ids_sorted),
                      _ptr(slotpos))
    return counts, offsets, ids_sorted, slotpos


def dequant_q4(codes, scales, biases):
    n = codes.shape[0]
    k = codes.shape[1] * 8
    out = np.zeros((n, k), np.uint16)
    lib().or_dequant_q4(_ptr(codes), _ptr(scales), _ptr(biases), n, k, _ptr(out))
    return out


def gemm_q4_grouped(a, w, counts, offsets, n_experts=64, with_acc=False):
    codes, scales, biases = w
    a = np.ascontiguousarray(a)
    S, K = a.shape
    N = codes.shape[0] // n_experts
    c = np.zeros((S, N), np.uint16)
    acc = np.zeros((S, N), np.float32) if with_acc else None
    lib().or_gemm_q4_grouped(_ptr(a), S, K, _ptr(codes), _ptr(scales), _ptr(biases), N,
                             _ptr(counts), _ptr(offsets), n_experts, _ptr(c), _ptr(acc))
    return (c, acc) if with_acc else c


def silu_mul(g, u):
    g = np.ascontiguousarray(g)
    u = np.ascontiguousarray(u)
    out = np.zeros_like(g)
    lib().or_silu_mul(_ptr(g), _ptr(u), C.c_size_t(g.size), _ptr(out))
    return out


def gather_rows(table, ids):
    table = np.ascontiguousarray(table)
    ids = np.ascontiguousarray(ids, dtype=np.uint32)
    H = table.shape[-1]
    out = np.zeros((ids.size, H), np.uint16)
    lib().or_gather_rows(_ptr(table), _ptr(ids), ids.size, H, _ptr(out))
    return out


def moe_combine(ed, slotpos, gw, m, H):
    out = np.zeros((m, H), np.uint16)
    lib().or_moe_combine(_ptr(np.ascontiguousarray(ed)), _ptr(np.ascontiguousarray(slotpos)),
                         _ptr(np.ascontiguousarray(gw)), m, 4, H, _ptr(out))
    return out


def moe_prefill(x, logits, gate, up, down, mode=0, bias=None, n_experts=64):
    """Returns dict(ids, gw, ids_sorted, slotpos, act, ed, out)."""
    x = np.ascontiguousarray(x)
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    m, H = x.shape
    I = gate[0].shape[0] // n_experts
    S = 4 * m
    r = dict(ids=np.zeros((m, 4), np.uint32), gw=np.zeros((m, 4), np.uint16),
             ids_sorted=np.zeros(S, np.uint32), slotpos=np.zeros(S, np.uint32),
             act=np.zeros((S, I), np.uint16), ed=np.zeros((S, H), np.uint16),
             out=np.zeros((m, H), np.uint16))
    lib().or_moe_prefill(_ptr(x), _ptr(logits), m, n_experts, H, I, mode, _ptr(bias),
                         *(_ptr(a) for a in gate), *(_ptr(a) for a in up),
                         *(_ptr(a) for a in down), _ptr(r["ids"]), _ptr(r["gw"]),
                         _ptr(r["ids_sorted"]), _ptr(r["slotpos"]), _ptr(r["act"]),
                         _ptr(r["ed"]), _ptr(r["out"]))
    return r


def proj3_gemv_scatter(q, k, v, x, v_cache, pos):
    """(q bf16 [nq], k bf16 [nk], the updated copy of v_cache bf16
    [nv/64][max_seq][64]) for weights q/k/v = (codes, scales, biases)."""
    nq, nk, nv = q[0].shape[0], k[0].shape[0], v[0].shape[0]
    K = q[0].shape[1] * 8
    x = np.ascontiguousarray(x.reshape(K))
    qo, ko = np.zeros(nq, np.uint16), np.zeros(nk, np.uint16)
    vc = np.ascontiguousarray(v_cache).copy()
    max_seq = vc.shape[1]
    lib().or_proj3_gemv_scatter(*(_ptr(a) for a in q), *(_ptr(a) for a in k),
                                *(_ptr(a) for a in v), nq, nk, nv, K, _ptr(x), _ptr(qo),
                                _ptr(ko), _ptr(vc), max_seq, pos)
    return qo, ko, vc


def conv3_gemv(w_proj, x, taps, state):
    """(out bf16 [H], new_state bf16 [2][H]) of the short conv for one row."""
    codes, scales, biases = w_proj
    H = codes.shape[0] // 3
    K = codes.shape[1] * 8
    out = np.zeros(H, np.uint16)
    ns = np.zeros((2, H), np.uint16)
    lib().or_conv3_gemv(_ptr(codes), _ptr(scales), _ptr(biases), H, K,
                        _ptr(np.ascontiguousarray(x.reshape(K))), _ptr(np.ascontiguousarray(taps)),
                        _ptr(np.ascontiguousarray(state)), _ptr(out), _ptr(ns))
    return out, ns


def gemv_gu_act(gate, up, x):
    """act bf16 [B][N] of the dense FFN front half."""
    N = gate[0].shape[0]
    K = gate[0].shape[1] * 8
    x = np.ascontiguousarray(x.reshape(-1, K))
    B = x.shape[0]
    act = np.zeros((B, N), np.uint16)
    lib().or_gemv_gu_act(*(_ptr(a) for a in gate), *(_ptr(a) for a in up), N, K, _ptr(x), B,
                         _ptr(act))
    return act


def sample_draw(logits, seen=None, temperature=1.0, top_k=0, top_p=1.0, penalty=1.0, seed=0,
                pos=0):
    """(argmax key u64, threshold key u32) of the sampled draw over bf16
    logits [V]; seen: u32 bitmap [V/32] or None."""
    logits = np.ascontiguousarray(logits.reshape(-1))
    V = logits.shape[0]
    tau = C.c_uint32(0)
    L = lib()
    L.or_sample_draw.restype = C.c_uint64
    L.or_sample_draw.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_float, C.c_uint32,
                                 C.c_float, C.c_float, C.c_uint64, C.c_uint32,
                                 C.POINTER(C.c_uint32)]
    key = L.or_sample_draw(_ptr(logits), V, _ptr(seen), temperature, top_k, top_p, penalty,
                           seed, pos, C.byref(tau))
    return int(key), int(tau.value)


def gumbel(x: int) -> float:
    L = lib()
    L.or_gumbel.restype = C.c_float
    L.or_gumbel.argtypes = [C.c_uint32]
    return L.or_gumbel(x)


def log(x: float) -> float:
    L = lib()
    L.or_log.restype = C.c_float
    L.or_log.argtypes = [C.c_float]
    return L.or_log(x)


def sample_word(i: int, pos: int, seed: int) -> int:
    L = lib()
    L.or_sample_word.restype = C.c_uint32
    L.or_sample_word.argtypes = [C.c_uint32] * 4
    return L.or_sample_word(i, pos, seed & 0xffffffff, seed >> 32)


def philox4x32_10(counter, key):
    """Philox4x32-10 of a 4-word counter and 2-word key -> 4 words."""
    c = (C.c_uint32 * 4)(*counter)
    L = lib()
    L.or_philox4x32_10.argtypes = [C.c_void_p, C.c_uint32, C.c_uint32]
    L.or_philox4x32_10(C.cast(c, C.c_void_p), key[0], key[1])
    return [int(v) for v in c]
