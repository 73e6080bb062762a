"""Op-level mirror of Molten's ``src/kernels/lfm.rs`` / ``elementwise.rs`` over the
CUDA C ABI.

Each function keeps the reference wrapper's name, argument meaning and
``ensure!``-style validation (raising ValueError before anything is
enqueued), then enqueues the sm_100a kernel on the context's stream. Tensors
are CUDA tensors owned by the caller; nothing here allocates device memory.
u32 buffers (ids, tokens, counters, codes) are int32 tensors holding the bit
patterns; the argmax key is an int64 tensor.
"""
from __future__ import annotations

import torch

from . import _lib
from .quant import QuantWeights, check_quant

ARGMAX_GROUPS = 64
FIXED_HIDDEN = 2048
FIXED_MOE_INTER = 1536
ROUTE_SOFTMAX_RENORM = _lib.ROUTE_SOFTMAX_RENORM
ROUTE_SIGMOID_BIAS = _lib.ROUTE_SIGMOID_BIAS
PREFILL_CHUNK = 256  # token rows per grouped-GEMM chunk (mc_moe_prefill's sort_map bm)
MOE_PREFILL_LAUNCHES = 7  # kernels one mc_moe_prefill call launches


def ensure(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def _p(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    ensure(t.is_cuda, "tensors must be on the GPU")
    ensure(t.is_contiguous(), "tensors must be contiguous")
    return t.data_ptr()


STATUS_BITS = {1: "a logits wait gave up", 2: "an expert id out of range",
               4: "rows beyond a capacity", 8: "an act wait gave up",
               16: "a copy wait gave up"}


def raise_on_status(word: torch.Tensor, what: str) -> None:
    """Reads a kernel status word (waits for the stream) and raises
    McError(MC_ETIMEOUT) if any bit is set: a bounded wait that ran out (or a
    malformed input the kernel skipped) means the outputs are not valid."""
    v = int(word.reshape(-1)[0].item()) & 0xffffffff
    if v:
        why = ", ".join(m for b, m in STATUS_BITS.items() if v & b) or "unknown bits"
        raise _lib.McError(_lib.MC_ETIMEOUT, f"{what}: status 0x{v:x} ({why})")


class Context:
    """MetalContext + ComputePass stand-in: one device and stream (metal.rs:91-400).

    By default work goes on torch's current stream of ``device`` at call time,
    so torch ops and these kernels interleave in order.
    """

    def __init__(self, device: int | torch.device = 0, stream: torch.cuda.Stream | None = None):
        dev = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        self.device = dev
        self._fixed_stream = stream
        h = _lib.C.c_void_p()
        s = (stream or torch.cuda.current_stream(dev)).cuda_stream
        _lib.check(_lib.lib().mc_create(dev.index or 0, s, _lib.C.byref(h)))
        self.h = h

    @property
    def handle(self):
        s = (self._fixed_stream or torch.cuda.current_stream(self.device)).cuda_stream
        _lib.check(_lib.lib().mc_set_stream(self.h, s))
        return self.h

    def commit_wait(self) -> None:
        _lib.check(_lib.lib().mc_sync(self.h))

    def prefetch_next(self, *tensors) -> None:
        """Cross-layer prefetch hint (mc_set_l2_prefetch, no reference
        counterpart): the next moe_decode_layer on this context pulls up to two
        tensors (e.g. the next layer's router and RMSNorm weights, or its
        router and projection codes) into L2."""
        ts = [t for t in tensors if t is not None][:2] + [None, None]
        args = []
        for t in ts[:2]:
            args += [t.data_ptr(), t.numel() * t.element_size()] if t is not None else [None, 0]
        _lib.check(_lib.lib().mc_set_l2_prefetch(self.h, *args))

    def set_wait_limit(self, ns: int) -> None:
        """Limit of every bounded device wait of later launches (0 = each
        kernel's default); a wait that runs out sets a status bit."""
        _lib.check(_lib.lib().mc_set_wait_limit(self.h, int(ns)))

    def set_test_flags(self, flags: int) -> None:
        """Test aid (mc_set_test_flags): 0 for normal work."""
        _lib.check(_lib.lib().mc_set_test_flags(self.h, int(flags)))

    def close(self) -> None:
        if self.h:
            _lib.lib().mc_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _bf16(*ts):
    for t in ts:
        if t is not None:
            ensure(t.dtype == torch.bfloat16, "expects BF16")


def _u32(*ts):
    for t in ts:
        if t is not None:
            ensure(t.dtype == torch.int32, "expects U32 (int32 storage)")


def copy_async(ctx: Context, dst: torch.Tensor, src: torch.Tensor) -> None:
    """Stream-ordered copy between device tensors and page-locked host tensors
    (Tensor::write_bytes / contents, tensor.rs:127-146, 165-200; on the GPU's
    own memory model the host rows are staged by the device). Same byte
    count, both contiguous; host tensors must be pinned."""
    for t in (dst, src):
        ensure(t.is_contiguous(), "copy_async: tensors must be contiguous")
        ensure(t.is_cuda or t.is_pinned(), "copy_async: host tensors must be pinned")
    nbytes = dst.numel() * dst.element_size()
    ensure(nbytes == src.numel() * src.element_size(), "copy_async: byte counts differ")
    _lib.call("mc_copy_async", ctx.handle, dst.data_ptr(), src.data_ptr(), nbytes)


# ----------------------------------------------------------------- decode ops

def gemv_quant(ctx: Context, w: QuantWeights, x: torch.Tensor, y: torch.Tensor) -> None:
    """gemv_quant (kernels/lfm.rs:112-149): y = W x for rows of x [batch, in]."""
    n, k = check_quant(w)
    ensure(x.shape[-1] == k and y.shape[-1] == n, "gemv shape mismatch")
    batch = x.numel() // k
    ensure(y.numel() == batch * n, "gemv shape mismatch")
    _bf16(x, y)
    _lib.call("mc_gemv_quant", ctx.handle, _lib.C.byref(w.qw()), _p(x), _p(y), batch)


def gemv_head_argmax(ctx: Context, w: QuantWeights, x: torch.Tensor, best: torch.Tensor) -> None:
    """gemv_head_argmax (kernels/lfm.rs:826-844): argmax keys folded into ``best``
    (int64 [batch], zero before the call)."""
    n, k = check_quant(w)
    batch = x.numel() // k
    ensure(x.numel() == batch * k and best.numel() >= batch and best.dtype == torch.int64,
           "head argmax input/key")
    _bf16(x)
    _lib.call("mc_gemv_head_argmax", ctx.handle, _lib.C.byref(w.qw()), _p(x), _p(best), batch)


def token_tail(ctx: Context, best: torch.Tensor, out_tok: torch.Tensor,
               next: tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor] | None = None,
               eps: float = 1e-5) -> None:
    """token_tail (kernels/lfm.rs:850-888). ``next = (embed, norm_w, x, normed)``
    with a bf16 embedding table [vocab, 2048]."""
    _u32(out_tok)
    batch = out_tok.numel()
    ensure(best.dtype == torch.int64 and best.numel() >= batch, "token tail key")
    if next is None:
        _lib.call("mc_token_tail", ctx.handle, _p(best), _p(out_tok), None, 0, None, None, None,
                  FIXED_HIDDEN, eps, batch)
        return
    embed, norm_w, x, normed = next
    _bf16(embed, norm_w, x, normed)
    ensure(embed.shape[-1] == FIXED_HIDDEN, "token tail embedding width")
    for t in (x, normed):
        ensure(t.numel() == batch * FIXED_HIDDEN, "token tail rows")
    _lib.call("mc_token_tail", ctx.handle, _p(best), _p(out_tok), _p(embed), embed.shape[0],
              _p(norm_w), _p(x), _p(normed), FIXED_HIDDEN, eps, batch)


def argmax_bf16(ctx: Context, x: torch.Tensor, out: torch.Tensor) -> None:
    """argmax_bf16 (kernels/lfm.rs:794-820) over rows of bf16 logits."""
    _bf16(x)
    _u32(out)
    n = x.shape[-1]
    batch = x.numel() // n
    ensure(out.numel() >= batch, "argmax output")
    _lib.call("mc_argmax_bf16", ctx.handle, _p(x), n, _p(out), batch)


def add_rmsnorm(ctx: Context, h: torch.Tensor, b: torch.Tensor | None, w: torch.Tensor,
                hout: torch.Tensor | None, out: torch.Tensor, eps: float = 1e-5) -> None:
    """add_rmsnorm_bf16 (norm.metal:63-136) for hidden 2048."""
    _bf16(h, b, w, hout, out)
    batch = h.numel() // FIXED_HIDDEN
    ensure(h.numel() == batch * FIXED_HIDDEN and out.numel() == h.numel(), "add_rmsnorm shapes")
    _lib.call("mc_add_rmsnorm", ctx.handle, _p(h), _p(b), _p(w), _p(hout), _p(out),
              FIXED_HIDDEN, eps, batch)


def router_addnorm_route(ctx: Context, h, b, nw, hout, normed, w, logits, bias, ids, weights,
                         counter, eps: float = 1e-5, route_mode: int = ROUTE_SOFTMAX_RENORM,
                         route_eps: float = 1e-6) -> None:
    """router_addnorm_route (kernels/lfm.rs:266-311). ``w`` is the [E, H] router
    in bf16 (BASELINE) or f32 (reference model); ``bias`` the f32 expert bias
    (used by the sigmoid mode, may be None)."""
    e, k = w.shape
    ensure(e <= 64 and k == FIXED_HIDDEN, "fused router route requires E<=64, H=2048")
    ensure(w.dtype in (torch.bfloat16, torch.float32), "router dtype")
    batch = h.numel() // k
    ensure(logits.numel() == batch * e and logits.dtype == torch.float32, "router logits shape")
    ensure(bias is None or (bias.numel() == e and bias.dtype == torch.float32), "router bias")
    for t in (h, b, hout, normed):
        ensure(t is None or t.numel() == batch * k, "router norm shapes")
    _bf16(h, b, nw, hout, normed, weights)
    _u32(ids, counter)
    ensure(ids.numel() == 4 * batch and weights.numel() == 4 * batch, "route outputs")
    ensure(counter.numel() >= batch, "route counter shape")
    dt = _lib.DTYPE_BF16 if w.dtype == torch.bfloat16 else _lib.DTYPE_F32
    _lib.call("mc_router_addnorm_route", ctx.handle, _p(h), _p(b), _p(nw), _p(hout), _p(normed),
              _p(w), dt, _p(bias), route_mode, _p(logits), _p(ids), _p(weights), _p(counter), e,
              k, eps, route_eps, batch)


def gemv_f32(ctx: Context, w: torch.Tensor, x: torch.Tensor, y: torch.Tensor) -> None:
    """gemv_f32 (kernels/lfm.rs:314-335): router logits y = W x (f32 out)."""
    e, k = w.shape
    batch = x.numel() // k
    ensure(y.numel() == batch * e and y.dtype == torch.float32, "gemv_f32 output F32")
    _bf16(x)
    dt = _lib.DTYPE_BF16 if w.dtype == torch.bfloat16 else _lib.DTYPE_F32
    _lib.call("mc_gemv_router", ctx.handle, _p(w), dt, _p(x), _p(y), e, k, batch)


def route_token(ctx: Context, logits, bias, ids, weights,
                route_mode: int = ROUTE_SOFTMAX_RENORM, route_eps: float = 1e-6) -> None:
    """route_token (kernels/lfm.rs:391-417)."""
    _u32(ids)
    _bf16(weights)
    batch = ids.numel() // 4
    e = logits.numel() // batch
    ensure(e <= 64 and logits.dtype == torch.float32, "router logits")
    _lib.call("mc_route_token", ctx.handle, _p(logits), e, route_mode, _p(bias), route_eps,
              _p(ids), _p(weights), batch)


def gemv_gather_act(ctx: Context, gate: QuantWeights, up: QuantWeights, x: torch.Tensor,
                    ids: torch.Tensor, act: torch.Tensor, n_experts: int = 64) -> None:
    """gemv_gather_act (kernels/lfm.rs:421-460)."""
    check_quant(gate)
    check_quant(up)
    k = x.shape[-1]
    batch = x.numel() // k
    n = gate.out_features // n_experts
    ensure(act.numel() == batch * 4 * n, "act shape")
    ensure(k == FIXED_HIDDEN and gate.in_features == k and up.in_features == k,
           "gather act is the compile-time expert shape")
    _bf16(x, act)
    _u32(ids)
    _lib.call("mc_gemv_gather_act", ctx.handle, _lib.C.byref(gate.qw()), _lib.C.byref(up.qw()),
              _p(x), _p(ids), _p(act), n_experts, batch)


def gemv_gather_down_combine4(ctx: Context, down: QuantWeights, act: torch.Tensor,
                              ids: torch.Tensor, weights: torch.Tensor, out: torch.Tensor,
                              n_experts: int = 64) -> None:
    """gemv_gather_down_combine4 (kernels/lfm.rs:499-533)."""
    check_quant(down)
    k = down.in_features
    n = down.out_features // n_experts
    batch = out.numel() // n
    ensure(act.numel() == batch * 4 * k and weights.numel() == batch * 4, "combine shapes")
    _bf16(act, weights, out)
    _u32(ids)
    _lib.call("mc_gemv_gather_down_combine4", ctx.handle, _lib.C.byref(down.qw()), _p(act),
              _p(ids), _p(weights), _p(out), n_experts, batch)


def proj3_gemv_scatter(ctx: Context, q: QuantWeights, k: QuantWeights, v: QuantWeights,
                       x: torch.Tensor, q_out: torch.Tensor, k_out: torch.Tensor,
                       v_cache: torch.Tensor, pos: int) -> None:
    """Decode-only Q, K, V projections in one launch, V written into the KV
    cache at ``pos`` (kernels/lfm.rs:150-205). v_cache: bf16
    [nv / 64, max_seq, 64]."""
    kdim = x.numel()
    nq, nk, nv = q.out_features, k.out_features, v.out_features
    ensure(q.in_features == kdim and k.in_features == kdim and v.in_features == kdim,
           "proj3 input width")
    ensure(q.bits == 4 and k.bits == 4 and v.bits == 4 and q.group_size == 64
           and k.group_size == 64 and v.group_size == 64, "proj3 is affine 4-bit/64")
    ensure(kdim == FIXED_HIDDEN, "proj3 input width is the compile-time hidden size")
    ensure(q_out.numel() == nq and k_out.numel() == nk and nv % 64 == 0, "proj3 output shape")
    _bf16(x, q_out, k_out, v_cache)
    ensure(v_cache.dim() == 3, "proj3 KV cache shape")
    max_seq = v_cache.shape[1]
    ensure(v_cache.shape[0] * 64 == nv and v_cache.shape[2] == 64 and 0 <= pos < max_seq,
           "proj3 KV cache shape")
    for w in (q, k, v):
        check_quant(w)
    _lib.call("mc_proj3_gemv_scatter", ctx.handle, _lib.C.byref(q.qw()), _lib.C.byref(k.qw()),
              _lib.C.byref(v.qw()), _p(x), _p(q_out), _p(k_out), _p(v_cache), max_seq, pos)


def conv3_gemv(ctx: Context, wproj: QuantWeights, x: torch.Tensor, w: torch.Tensor,
               state: torch.Tensor, out: torch.Tensor, new_state: torch.Tensor) -> None:
    """Decode-only short-conv B/C/X projection and the conv in one launch
    (kernels/lfm.rs:207-246). w: taps bf16 [H, 3]; state, new_state bf16 [2, H]."""
    kdim, h = x.numel(), out.numel()
    ensure(wproj.out_features == 3 * h and wproj.in_features == kdim, "conv3 projection shape")
    ensure(wproj.bits == 4 and wproj.group_size == 64, "conv3 projection 4-bit/64")
    ensure(kdim == FIXED_HIDDEN, "conv3 input width is the compile-time hidden size")
    ensure(w.numel() == 3 * h, "conv3 tap shape")
    ensure(tuple(state.shape) == (2, h) and tuple(new_state.shape) == (2, h), "conv3 state shape")
    _bf16(x, w, state, out, new_state)
    check_quant(wproj)
    _lib.call("mc_conv3_gemv", ctx.handle, _lib.C.byref(wproj.qw()), _p(x), _p(w), _p(state),
              _p(out), _p(new_state), h)


def gemv_gu_act(ctx: Context, gate: QuantWeights, up: QuantWeights, x: torch.Tensor,
                act: torch.Tensor) -> None:
    """Decode dense FFN front half, act = silu(x gate^T) * (x up^T) with the
    separate GEMVs' bf16 roundings (kernels/lfm.rs:462-495). x [B, K] (or
    [K]), act [B, N]."""
    n, k = gate.out_features, gate.in_features
    ensure(gate.bits == 4 and up.bits == 4, "dense gate/up must be 4-bit")
    ensure(up.out_features == n and up.in_features == k and up.group_size == gate.group_size,
           "dense gate/up shapes")
    ensure(x.numel() % k == 0 and act.numel() == (x.numel() // k) * n, "dense gate/up rows")
    _bf16(x, act)
    for w in (gate, up):
        check_quant(w)
    _lib.call("mc_gemv_gu_act", ctx.handle, _lib.C.byref(gate.qw()), _lib.C.byref(up.qw()),
              _p(x), _p(act), x.numel() // k)


def moe_decode_workspace_words(moe_inter: int = FIXED_MOE_INTER) -> int:
    """u32 words of workspace moe_decode_layer needs (zero it once)."""
    return int(_lib.lib().mc_moe_decode_workspace_words(moe_inter))


def moe_decode_layer(ctx: Context, h, b, nw, hout, normed, router, logits, bias, ids, weights,
                     gate: QuantWeights, up: QuantWeights, down: QuantWeights, out, workspace,
                     eps: float = 1e-5, route_mode: int = ROUTE_SOFTMAX_RENORM,
                     route_eps: float = 1e-6, n_experts: int = 64, check: bool = False) -> None:
    """moe_decode (lfm.rs:967-1011) with the fused router, one persistent launch
    for one token. ``workspace``: int32 [moe_decode_workspace_words(I)], zeroed
    once, then reused by one chain of calls (it carries an epoch; its word 2
    is the sticky status). ``check``: wait for the launch and raise McError
    if the status word is nonzero."""
    for w in (gate, up, down):
        check_quant(w)
    e, k = router.shape
    ensure(e == n_experts and k == FIXED_HIDDEN, "router shape")
    ensure(h.numel() == k and out.numel() == k, "moe_decode_layer is batch 1")
    _bf16(h, b, nw, hout, normed, weights, out)
    _u32(ids, workspace)
    dt = _lib.DTYPE_BF16 if router.dtype == torch.bfloat16 else _lib.DTYPE_F32
    _lib.call("mc_moe_decode_layer", ctx.handle, _p(h), _p(b), _p(nw), _p(hout), _p(normed),
              _p(router), dt, _p(bias), route_mode, _p(logits), _p(ids), _p(weights),
              _lib.C.byref(gate.qw()), _lib.C.byref(up.qw()), _lib.C.byref(down.qw()),
              n_experts, _p(out), _p(workspace), workspace.numel(), eps, route_eps)
    if check:
        raise_on_status(workspace[2:3], "moe_decode_layer")


def moe_decode_layer_noalloc(ctx: Context, h, b, nw, hout, normed, router, logits, bias, ids,
                             weights, gate: QuantWeights, up: QuantWeights, down: QuantWeights,
                             out, status=None, eps: float = 1e-5,
                             route_mode: int = ROUTE_SOFTMAX_RENORM, route_eps: float = 1e-6,
                             n_experts: int = 64, check: bool = False) -> None:
    """moe_decode_layer with the library's built-in per-device scratch instead
    of a caller workspace (expert width <= 2048). The first call per device
    sets the scratch up and blocks; calls that could overlap on one device
    race. ``status``: optional int32 [1] receiving this call's status word;
    ``check`` (needs ``status``) waits and raises McError if it is nonzero."""
    ensure(not check or status is not None, "check needs a status word")
    for w in (gate, up, down):
        check_quant(w)
    e, k = router.shape
    ensure(e == n_experts and k == FIXED_HIDDEN, "router shape")
    ensure(h.numel() == k and out.numel() == k, "moe_decode_layer_noalloc is batch 1")
    _bf16(h, b, nw, hout, normed, weights, out)
    _u32(ids, status)
    dt = _lib.DTYPE_BF16 if router.dtype == torch.bfloat16 else _lib.DTYPE_F32
    _lib.call("mc_moe_decode_layer_noalloc", ctx.handle, _p(h), _p(b), _p(nw), _p(hout),
              _p(normed), _p(router), dt, _p(bias), route_mode, _p(logits), _p(ids), _p(weights),
              _lib.C.byref(gate.qw()), _lib.C.byref(up.qw()), _lib.C.byref(down.qw()),
              n_experts, _p(out), _p(status), eps, route_eps)
    if check:
        raise_on_status(status, "moe_decode_layer_noalloc")


def moe_decode_proj_workspace_words(moe_inter: int = FIXED_MOE_INTER) -> int:
    """u32 words of workspace moe_decode_layer_proj needs (zero it once)."""
    return int(_lib.lib().mc_moe_decode_proj_workspace_words(moe_inter))


def moe_decode_layer_proj(ctx: Context, h, proj: QuantWeights, nw, hout, normed, router, logits,
                          bias, ids, weights, gate: QuantWeights, up: QuantWeights,
                          down: QuantWeights, out, workspace, p_out=None, eps: float = 1e-5,
                          route_mode: int = ROUTE_SOFTMAX_RENORM, route_eps: float = 1e-6,
                          n_experts: int = 64, check: bool = False) -> None:
    """gemv_quant(proj, h) -> b (kernels/lfm.rs:112-149) and moe_decode_layer(h,
    b, ...) in one launch, bit-identical to the two calls. ``workspace``:
    int32 [moe_decode_proj_workspace_words(I)], zeroed once, owned by one
    chain of calls; ``p_out`` (optional bf16 [2048]) receives b."""
    for w in (proj, gate, up, down):
        check_quant(w)
    ensure(proj.bits == 4 and proj.in_features == FIXED_HIDDEN and
           proj.out_features == FIXED_HIDDEN, "proj must be Q4 2048 x 2048")
    e, k = router.shape
    ensure(e == n_experts and k == FIXED_HIDDEN, "router shape")
    ensure(h.numel() == k and out.numel() == k, "moe_decode_layer_proj is batch 1")
    ensure(p_out is None or p_out.numel() == k, "p_out shape")
    _bf16(h, nw, hout, normed, weights, out)
    if p_out is not None:
        _bf16(p_out)
    _u32(ids, workspace)
    dt = _lib.DTYPE_BF16 if router.dtype == torch.bfloat16 else _lib.DTYPE_F32
    _lib.call("mc_moe_decode_layer_proj", ctx.handle, _p(h), _lib.C.byref(proj.qw()),
              _p(p_out), _p(nw), _p(hout), _p(normed), _p(router), dt, _p(bias), route_mode,
              _p(logits), _p(ids), _p(weights), _lib.C.byref(gate.qw()), _lib.C.byref(up.qw()),
              _lib.C.byref(down.qw()), n_experts, _p(out), _p(workspace), workspace.numel(), eps,
              route_eps)
    if check:
        raise_on_status(workspace[2:3], "moe_decode_layer_proj")


def decode_workspace_act(workspace: torch.Tensor, moe_inter: int = FIXED_MOE_INTER):
    """The act rows (bf16 [4, I]) held in a moe_decode_layer workspace: one
    tagged word per value (tag << 16 | bf16 bits), little-endian, so the low
    16-bit halves are the values."""
    w = workspace[136:136 + 4 * moe_inter].contiguous().view(torch.int16)[0::2].contiguous()
    return w.view(torch.bfloat16).reshape(4, moe_inter)


# ---------------------------------------------------------------- prefill ops

def moe_route_batch(ctx: Context, logits, bias, ids, gw, m: int,
                    route_mode: int = ROUTE_SOFTMAX_RENORM, route_eps: float = 1e-6) -> None:
    """moe_route_batch (kernels/lfm.rs:536-555)."""
    e = logits.numel() // m
    ensure(ids.numel() == m * 4 and gw.numel() == m * 4, "route batch shapes")
    _u32(ids)
    _bf16(gw)
    _lib.call("mc_moe_route_batch", ctx.handle, _p(logits), m, e, route_mode, _p(bias),
              route_eps, _p(ids), _p(gw))


def moe_sort_map(ctx: Context, ids, counts, offsets, ids_sorted, slotpos, tiles, n_tiles,
                 m: int, bm: int = 128) -> None:
    """moe_zero_counts .. moe_blocks (kernels/lfm.rs:557-697) in two launches."""
    e = counts.numel()
    _u32(ids, counts, offsets, ids_sorted, slotpos, tiles, n_tiles)
    ensure(tiles.numel() % 4 == 0, "tile list is uint4 entries")
    _lib.call("mc_moe_sort_map", ctx.handle, _p(ids), m, e, bm, _p(counts), _p(offsets),
              _p(ids_sorted), _p(slotpos), _p(tiles), _p(n_tiles), tiles.numel() // 4)


def gather_rows_bf16(ctx: Context, table: torch.Tensor, ids: torch.Tensor,
                     out: torch.Tensor) -> None:
    """gather_rows_bf16 (elementwise.rs:59-104)."""
    _bf16(table, out)
    _u32(ids)
    h = table.shape[-1]
    ensure(out.numel() == ids.numel() * h, "gather out shape")
    _lib.call("mc_gather_rows_bf16", ctx.handle, _p(table), _p(ids), ids.numel(), h, _p(out))


def gemm_q4_grouped(ctx: Context, a: torch.Tensor, w: QuantWeights, c: torch.Tensor,
                    tiles: torch.Tensor, n_tiles: torch.Tensor, n_experts: int = 64,
                    status: torch.Tensor | None = None) -> None:
    """gemm_q4_grouped_mlx (quant.rs:228-266): tcgen05 grouped Q4 GEMM over the
    row tiles of moe_sort_map (bm = 128)."""
    check_quant(w)
    rows, k = a.shape
    ensure(k == w.in_features and c.shape[0] == rows, "grouped GEMM shapes")
    _bf16(a, c)
    _u32(tiles, n_tiles, status)
    _lib.call("mc_gemm_q4_grouped", ctx.handle, _p(a), rows, _lib.C.byref(w.qw()), n_experts,
              _p(c), _p(tiles), _p(n_tiles), tiles.numel() // 4, _p(status))


def gemm_q4_workspace_words(m: int) -> int:
    return int(_lib.lib().mc_gemm_q4_workspace_words(m))


def gemm_q4(ctx: Context, a: torch.Tensor, w: QuantWeights, c: torch.Tensor,
            workspace: torch.Tensor, status: torch.Tensor | None = None) -> None:
    """dequant_q4_bf16_bulk + gemm_bf16_nt (quant.metal:69-114, gemm.rs:33-60;
    the prefill projections of lfm.rs:661-671): c = a . bf16(W)^T on the
    tensor cores, W dequantised on the fly. workspace: int32
    [gemm_q4_workspace_words(m)]."""
    check_quant(w)
    m, k = a.shape
    ensure(k == w.in_features and tuple(c.shape) == (m, w.out_features), "gemm_q4 shapes")
    _bf16(a, c)
    _u32(workspace, status)
    _lib.call("mc_gemm_q4", ctx.handle, _p(a), m, _lib.C.byref(w.qw()), _p(c), _p(workspace),
              workspace.numel(), _p(status))


def gemm_q4_grouped_gu(ctx: Context, a: torch.Tensor, gate: QuantWeights, up: QuantWeights,
                       act: torch.Tensor, tiles: torch.Tensor, n_tiles: torch.Tensor,
                       n_experts: int = 64, status: torch.Tensor | None = None) -> None:
    """gemm_q4_grouped_mlx_gu + silu_mul_bf16 (quant.rs:146-199): gate and up
    grouped GEMMs sharing the A tile, SwiGLU in the epilogue."""
    check_quant(gate)
    check_quant(up)
    rows, k = a.shape
    ensure(k == gate.in_features and act.shape[0] == rows, "grouped gate/up shapes")
    _bf16(a, act)
    _u32(tiles, n_tiles, status)
    _lib.call("mc_gemm_q4_grouped_gu", ctx.handle, _p(a), rows, _lib.C.byref(gate.qw()),
              _lib.C.byref(up.qw()), n_experts, _p(act), _p(tiles), _p(n_tiles),
              tiles.numel() // 4, _p(status))


def silu_mul_bf16(ctx: Context, gate: torch.Tensor, up: torch.Tensor, out: torch.Tensor) -> None:
    """silu_mul_bf16 (elementwise.rs:48-56)."""
    _bf16(gate, up, out)
    ensure(gate.numel() == up.numel() == out.numel(), "size mismatch in silu_mul_bf16")
    _lib.call("mc_silu_mul_bf16", ctx.handle, _p(gate), _p(up), _p(out), gate.numel())


def moe_combine_rows(ctx: Context, sorted_rows, slotpos, weights, out, topk: int = 4) -> None:
    """moe_combine_rows (kernels/lfm.rs:701-756)."""
    m, h = out.shape
    ensure(sorted_rows.shape[-1] == h and sorted_rows.numel() >= m * topk * h,
           "combine sorted shape")
    _bf16(sorted_rows, weights, out)
    _u32(slotpos)
    _lib.call("mc_moe_combine_rows", ctx.handle, _p(sorted_rows), _p(slotpos), _p(weights),
              _p(out), m, topk, h)


def eval_math(ctx: Context, op: int, x: torch.Tensor, y: torch.Tensor) -> None:
    """Device math probe (0 exp, 1 silu, 2 sigmoid, 3 bf16 rounding)."""
    ensure(x.dtype == torch.float32 and y.dtype == torch.float32, "f32 only")
    _lib.call("mc_eval_math", ctx.handle, op, _p(x), _p(y), x.numel())


def moe_prefill_workspace_size(m: int, n_experts: int = 64, hidden: int = FIXED_HIDDEN,
                               moe_inter: int = FIXED_MOE_INTER) -> int:
    return int(_lib.lib().mc_moe_prefill_workspace_size(m, n_experts, hidden, moe_inter))


def moe_prefill(ctx: Context, x: torch.Tensor, logits: torch.Tensor, gate: QuantWeights,
                up: QuantWeights, down: QuantWeights, workspace: torch.Tensor, out: torch.Tensor,
                n_experts: int = 64, route_mode: int = ROUTE_SOFTMAX_RENORM,
                bias: torch.Tensor | None = None, check: bool = False) -> None:
    """moe_prefill (lfm.rs:847-965) from the router logits on, all on device.
    ``check``: wait and raise McError if the grouped GEMMs' status word (in
    the workspace) is nonzero."""
    for w in (gate, up, down):
        check_quant(w)
    m, h = x.shape
    ensure(logits.shape == (m, n_experts) and logits.dtype == torch.float32, "prefill logits")
    ensure(out.shape == (m, h), "prefill out shape")
    _bf16(x, out)
    ensure(workspace.dtype == torch.uint8, "workspace is a byte tensor")
    _lib.call("mc_moe_prefill", ctx.handle, _p(x), _p(logits), m, _lib.C.byref(gate.qw()),
              _lib.C.byref(up.qw()), _lib.C.byref(down.qw()), n_experts, route_mode, _p(bias),
              _p(workspace), workspace.numel(), _p(out))
    if check:
        I = gate.out_features // n_experts
        raise_on_status(prefill_workspace_view(workspace, m, n_experts, h, I)["status"],
                        "moe_prefill")


def prefill_workspace_view(workspace: torch.Tensor, m: int, n_experts: int = 64,
                           hidden: int = FIXED_HIDDEN, moe_inter: int = FIXED_MOE_INTER) -> dict:
    """Named views of a moe_prefill workspace (layout of moe_prefill.cu)."""
    S = 4 * m
    al = lambda v: (v + 255) & ~255
    offs, o = {}, 0
    max_tiles = (S + PREFILL_CHUNK - 1) // PREFILL_CHUNK + n_experts
    for name, nbytes in (("ids", S * 4), ("gw", S * 2), ("counts", n_experts * 4),
                         ("offsets", n_experts * 4), ("ids_sorted", S * 4), ("slotpos", S * 4),
                         ("tiles", max_tiles * 16), ("ctl", 8), ("gx", S * hidden * 2),
                         ("act", S * moe_inter * 2), ("ed", S * hidden * 2)):
        offs[name] = (o, nbytes)
        o = al(o + nbytes)
    v = {k: workspace[a:a + n] for k, (a, n) in offs.items()}
    u32 = lambda t: t.view(torch.int32)
    b16 = lambda t: t.view(torch.bfloat16)
    return dict(ids=u32(v["ids"]).view(m, 4), gw=b16(v["gw"]).view(m, 4),
                ids_sorted=u32(v["ids_sorted"]), slotpos=u32(v["slotpos"]),
                status=u32(v["ctl"])[1:2], n_tiles=u32(v["ctl"])[0:1],
                tiles=u32(v["tiles"]).view(max_tiles, 4), gx=b16(v["gx"]).view(S, hidden),
                act=b16(v["act"]).view(S, moe_inter), ed=b16(v["ed"]).view(S, hidden))
