//! `src/cuda.rs` for Molten: the extern "C" declarations of the B200 CUDA
//! backend (libmolten_cuda.so, include/molten_cuda.h), one per entry point,
//! for the Rust host to call in place of the Metal dispatches of
//! src/kernels/{lfm,quant,elementwise}.rs and src/lfm/sample.rs. Pointers are
//! device pointers (mc_copy_async also takes page-locked host memory); bf16
//! values travel as u16 bit patterns; every call returns 0 or a negative
//! MC_E* code with the message in mc_last_error(). The op-level wrappers with
//! the reference's `ensure!` checks follow the pattern `check(unsafe {
//! mc_gemv_quant(...) })`; tests/test_rust_binding.py checks every
//! declaration below against the C header.
#![allow(non_camel_case_types, dead_code)]

use std::ffi::CStr;
use std::os::raw::{c_char, c_int, c_void};

pub const MC_OK: c_int = 0;
pub const MC_EINVAL: c_int = -1;
pub const MC_ECUDA: c_int = -2;
pub const MC_EUNSUPPORTED: c_int = -3;
pub const MC_ENCCL: c_int = -4;
pub const MC_ETIMEOUT: c_int = -5;
pub const MC_ROUTE_SOFTMAX_RENORM: c_int = 0;
pub const MC_ROUTE_SIGMOID_BIAS: c_int = 1;
pub const MC_DTYPE_BF16: c_int = 0;
pub const MC_DTYPE_F32: c_int = 1;
pub const MC_TEST_SKIP_LOGIT_PUBLISH: c_int = 1;
pub const MC_TEST_SKIP_BARRIER_ARRIVE: c_int = 2;

/// mc_ctx: opaque (one device and stream; expert-parallel state).
#[repr(C)]
pub struct McCtx {
    _private: [u8; 0],
}

/// mc_qweights (weights.rs:11-30): device pointers, caller-owned.
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct McQweights {
    pub codes: *const u32,
    pub scales: *const u16,
    pub biases: *const u16,
    pub out_features: i32,
    pub in_features: i32,
    pub group_size: i32,
    pub bits: i32,
}

/// mc_sampling (lfm/sample.rs Sampling).
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct McSampling {
    pub temperature: f32,
    pub top_k: u32,
    pub top_p: f32,
    pub repetition_penalty: f32,
    pub seed: u64,
}

#[link(name = "molten_cuda")]
extern "C" {
    pub fn mc_create(device: c_int, stream: *mut c_void, out: *mut *mut McCtx) -> c_int;
    pub fn mc_destroy(ctx: *mut McCtx) -> c_int;
    pub fn mc_set_stream(ctx: *mut McCtx, stream: *mut c_void) -> c_int;
    pub fn mc_sync(ctx: *mut McCtx) -> c_int;
    pub fn mc_last_error() -> *const c_char;
    pub fn mc_version() -> *const c_char;
    pub fn mc_check_quant(w: *const McQweights) -> c_int;
    pub fn mc_gemv_quant(
        ctx: *mut McCtx,
        w: *const McQweights,
        x: *const u16,
        y: *mut u16,
        batch: c_int,
    ) -> c_int;
    pub fn mc_gemv_head_argmax(
        ctx: *mut McCtx,
        w: *const McQweights,
        x: *const u16,
        keys: *mut u64,
        batch: c_int,
    ) -> c_int;
    pub fn mc_token_tail(
        ctx: *mut McCtx,
        keys: *mut u64,
        out_tok: *mut u32,
        embed: *const u16,
        vocab: c_int,
        norm_w: *const u16,
        x_next: *mut u16,
        normed_next: *mut u16,
        hidden: c_int,
        eps: f32,
        batch: c_int,
    ) -> c_int;
    pub fn mc_argmax_bf16(
        ctx: *mut McCtx,
        logits: *const u16,
        n: c_int,
        out: *mut u32,
        batch: c_int,
    ) -> c_int;
    pub fn mc_add_rmsnorm(
        ctx: *mut McCtx,
        h: *const u16,
        b: *const u16,
        w: *const u16,
        hout: *mut u16,
        nout: *mut u16,
        hidden: c_int,
        eps: f32,
        batch: c_int,
    ) -> c_int;
    pub fn mc_router_addnorm_route(
        ctx: *mut McCtx,
        h: *const u16,
        b: *const u16,
        norm_w: *const u16,
        h_out: *mut u16,
        normed: *mut u16,
        router_w: *const c_void,
        router_dtype: c_int,
        expert_bias: *const f32,
        route_mode: c_int,
        logits: *mut f32,
        ids: *mut u32,
        weights: *mut u16,
        counter: *mut u32,
        n_experts: c_int,
        hidden: c_int,
        eps: f32,
        route_eps: f32,
        batch: c_int,
    ) -> c_int;
    pub fn mc_gemv_router(
        ctx: *mut McCtx,
        router_w: *const c_void,
        router_dtype: c_int,
        x: *const u16,
        logits: *mut f32,
        n_experts: c_int,
        hidden: c_int,
        batch: c_int,
    ) -> c_int;
    pub fn mc_route_token(
        ctx: *mut McCtx,
        logits: *const f32,
        n_experts: c_int,
        route_mode: c_int,
        expert_bias: *const f32,
        route_eps: f32,
        ids: *mut u32,
        weights: *mut u16,
        batch: c_int,
    ) -> c_int;
    pub fn mc_gemv_gather_act(
        ctx: *mut McCtx,
        gate: *const McQweights,
        up: *const McQweights,
        x: *const u16,
        ids: *const u32,
        act: *mut u16,
        n_experts: c_int,
        batch: c_int,
    ) -> c_int;
    pub fn mc_gemv_gather_down_combine4(
        ctx: *mut McCtx,
        down: *const McQweights,
        act: *const u16,
        ids: *const u32,
        weights: *const u16,
        out: *mut u16,
        n_experts: c_int,
        batch: c_int,
    ) -> c_int;
    pub fn mc_moe_decode_workspace_words(moe_inter: c_int) -> usize;
    pub fn mc_moe_decode_layer(
        ctx: *mut McCtx,
        h: *const u16,
        b: *const u16,
        norm_w: *const u16,
        h_out: *mut u16,
        normed: *mut u16,
        router_w: *const c_void,
        router_dtype: c_int,
        expert_bias: *const f32,
        route_mode: c_int,
        logits: *mut f32,
        ids: *mut u32,
        weights: *mut u16,
        gate: *const McQweights,
        up: *const McQweights,
        down: *const McQweights,
        n_experts: c_int,
        out: *mut u16,
        workspace: *mut u32,
        ws_words: usize,
        eps: f32,
        route_eps: f32,
    ) -> c_int;
    pub fn mc_moe_decode_layer_noalloc(
        ctx: *mut McCtx,
        h: *const u16,
        b: *const u16,
        norm_w: *const u16,
        h_out: *mut u16,
        normed: *mut u16,
        router_w: *const c_void,
        router_dtype: c_int,
        expert_bias: *const f32,
        route_mode: c_int,
        logits: *mut f32,
        ids: *mut u32,
        weights: *mut u16,
        gate: *const McQweights,
        up: *const McQweights,
        down: *const McQweights,
        n_experts: c_int,
        out: *mut u16,
        status: *mut u32,
        eps: f32,
        route_eps: f32,
    ) -> c_int;
    pub fn mc_moe_decode_proj_workspace_words(moe_inter: c_int) -> usize;
    pub fn mc_moe_decode_layer_proj(
        ctx: *mut McCtx,
        h: *const u16,
        proj: *const McQweights,
        p_out: *mut u16,
        norm_w: *const u16,
        h_out: *mut u16,
        normed: *mut u16,
        router_w: *const c_void,
        router_dtype: c_int,
        expert_bias: *const f32,
        route_mode: c_int,
        logits: *mut f32,
        ids: *mut u32,
        weights: *mut u16,
        gate: *const McQweights,
        up: *const McQweights,
        down: *const McQweights,
        n_experts: c_int,
        out: *mut u16,
        workspace: *mut u32,
        ws_words: usize,
        eps: f32,
        route_eps: f32,
    ) -> c_int;
    pub fn mc_proj3_gemv_scatter(
        ctx: *mut McCtx,
        q: *const McQweights,
        k: *const McQweights,
        v: *const McQweights,
        x: *const u16,
        q_out: *mut u16,
        k_out: *mut u16,
        v_cache: *mut u16,
        max_seq: c_int,
        pos: c_int,
    ) -> c_int;
    pub fn mc_conv3_gemv(
        ctx: *mut McCtx,
        w_proj: *const McQweights,
        x: *const u16,
        taps: *const u16,
        state: *const u16,
        out: *mut u16,
        new_state: *mut u16,
        channels: c_int,
    ) -> c_int;
    pub fn mc_gemv_gu_act(
        ctx: *mut McCtx,
        gate: *const McQweights,
        up: *const McQweights,
        x: *const u16,
        act: *mut u16,
        batch: c_int,
    ) -> c_int;
    pub fn mc_sample_workspace_bytes(vocab: c_int) -> usize;
    pub fn mc_sample_draw(
        ctx: *mut McCtx,
        logits: *const u16,
        vocab: c_int,
        seen: *const u32,
        s: *const McSampling,
        pos: u32,
        pos_dev: *const u32,
        key: *mut u64,
        workspace: *mut c_void,
        ws_bytes: usize,
    ) -> c_int;
    pub fn mc_sample_mark(ctx: *mut McCtx, tok: *const u32, seen: *mut u32, vocab: c_int, pos_dev: *mut u32) -> c_int;
    pub fn mc_moe_route_batch(
        ctx: *mut McCtx,
        logits: *const f32,
        m: c_int,
        n_experts: c_int,
        route_mode: c_int,
        expert_bias: *const f32,
        route_eps: f32,
        ids: *mut u32,
        gw: *mut u16,
    ) -> c_int;
    pub fn mc_moe_sort_map(
        ctx: *mut McCtx,
        ids: *const u32,
        m: c_int,
        n_experts: c_int,
        bm: c_int,
        counts: *mut u32,
        offsets: *mut u32,
        ids_sorted: *mut u32,
        slotpos: *mut u32,
        tiles: *mut u32,
        n_tiles: *mut u32,
        max_tiles: c_int,
    ) -> c_int;
    pub fn mc_gather_rows_bf16(
        ctx: *mut McCtx,
        table: *const u16,
        ids: *const u32,
        rows: c_int,
        hidden: c_int,
        out: *mut u16,
    ) -> c_int;
    pub fn mc_gemm_q4_workspace_words(m: c_int) -> usize;
    pub fn mc_gemm_q4(
        ctx: *mut McCtx,
        a: *const u16,
        m: c_int,
        w: *const McQweights,
        c: *mut u16,
        workspace: *mut u32,
        ws_words: usize,
        status: *mut u32,
    ) -> c_int;
    pub fn mc_gemm_q4_grouped(
        ctx: *mut McCtx,
        a: *const u16,
        rows: c_int,
        w: *const McQweights,
        n_experts: c_int,
        c: *mut u16,
        tiles: *const u32,
        n_tiles: *const u32,
        max_tiles: c_int,
        status: *mut u32,
    ) -> c_int;
    pub fn mc_gemm_q4_grouped_gu(
        ctx: *mut McCtx,
        a: *const u16,
        rows: c_int,
        gate: *const McQweights,
        up: *const McQweights,
        n_experts: c_int,
        act: *mut u16,
        tiles: *const u32,
        n_tiles: *const u32,
        max_tiles: c_int,
        status: *mut u32,
    ) -> c_int;
    pub fn mc_silu_mul_bf16(
        ctx: *mut McCtx,
        gate: *const u16,
        up: *const u16,
        out: *mut u16,
        n: usize,
    ) -> c_int;
    pub fn mc_moe_combine_rows(
        ctx: *mut McCtx,
        ed: *const u16,
        slotpos: *const u32,
        gw: *const u16,
        out: *mut u16,
        m: c_int,
        topk: c_int,
        hidden: c_int,
    ) -> c_int;
    pub fn mc_moe_prefill_workspace_size(
        m: c_int,
        n_experts: c_int,
        hidden: c_int,
        moe_inter: c_int,
    ) -> usize;
    pub fn mc_moe_prefill(
        ctx: *mut McCtx,
        x: *const u16,
        logits: *const f32,
        m: c_int,
        gate: *const McQweights,
        up: *const McQweights,
        down: *const McQweights,
        n_experts: c_int,
        route_mode: c_int,
        expert_bias: *const f32,
        workspace: *mut c_void,
        ws_bytes: usize,
        out: *mut u16,
    ) -> c_int;
    pub fn mc_map_ids(
        ctx: *mut McCtx,
        ids: *mut u32,
        n: usize,
        table: *const u32,
        n_experts: c_int,
        status: *mut u32,
    ) -> c_int;
    pub fn mc_ep_alloc(ctx: *mut McCtx, bytes: usize, out: *mut *mut c_void) -> c_int;
    pub fn mc_ep_free(ctx: *mut McCtx, ptr: *mut c_void) -> c_int;
    pub fn mc_ipc_handle(ctx: *mut McCtx, base: *mut c_void, handle_out: *mut c_void) -> c_int;
    pub fn mc_ipc_open(ctx: *mut McCtx, handle: *const c_void, out: *mut *mut c_void) -> c_int;
    pub fn mc_ipc_close(ctx: *mut McCtx, ptr: *mut c_void) -> c_int;
    pub fn mc_ep_dispatch(
        ctx: *mut McCtx,
        x: *const u16,
        m: c_int,
        hidden: c_int,
        ids_sorted: *const u32,
        counts_all: *const u32,
        rank: c_int,
        world: c_int,
        n_experts: c_int,
        recv_bufs: *const *mut c_void,
        recv_cap_rows: usize,
        status: *mut u32,
    ) -> c_int;
    pub fn mc_ep_tiles(
        ctx: *mut McCtx,
        counts_all: *const u32,
        rank: c_int,
        world: c_int,
        n_experts: c_int,
        bm: c_int,
        tiles: *mut u32,
        n_tiles: *mut u32,
        rows: *mut u32,
        max_tiles: c_int,
    ) -> c_int;
    pub fn mc_ep_return(
        ctx: *mut McCtx,
        ed: *const u16,
        ed_rows: usize,
        hidden: c_int,
        counts_all: *const u32,
        rank: c_int,
        world: c_int,
        n_experts: c_int,
        home_bufs: *const *mut c_void,
        home_cap_rows: usize,
        status: *mut u32,
    ) -> c_int;
    pub fn mc_ep_unique_id(out128: *mut c_void) -> c_int;
    pub fn mc_ep_init(
        ctx: *mut McCtx,
        nranks: c_int,
        rank: c_int,
        nccl_unique_id: *const c_void,
        timeout_ms: c_int,
    ) -> c_int;
    pub fn mc_ep_reserve(
        ctx: *mut McCtx,
        m_max: c_int,
        n_experts: c_int,
        slots_per_rank: c_int,
        hidden: c_int,
        moe_inter: c_int,
    ) -> c_int;
    pub fn mc_ep_place(
        load: *const u64,
        world: c_int,
        n_experts: c_int,
        slots_per_rank: c_int,
        tables: *mut u32,
        slot_expert: *mut i32,
    ) -> c_int;
    pub fn mc_ep_moe_prefill(
        ctx: *mut McCtx,
        x: *const u16,
        logits: *const f32,
        m: c_int,
        gate: *const McQweights,
        up: *const McQweights,
        down: *const McQweights,
        slot_table: *const u32,
        route_mode: c_int,
        expert_bias: *const f32,
        out: *mut u16,
    ) -> c_int;
    pub fn mc_ep_status(ctx: *mut McCtx, out: *mut u32) -> c_int;
    pub fn mc_ep_counts(ctx: *mut McCtx, out: *mut u32, n: usize) -> c_int;
    pub fn mc_ep_finalize(ctx: *mut McCtx) -> c_int;
    pub fn mc_ep_set_profile(ctx: *mut McCtx, on: c_int) -> c_int;
    pub fn mc_ep_phase_ms(ctx: *mut McCtx, out7: *mut f32) -> c_int;
    pub fn mc_set_l2_prefetch(
        ctx: *mut McCtx,
        p0: *const c_void,
        n0: usize,
        p1: *const c_void,
        n1: usize,
    ) -> c_int;
    pub fn mc_copy_async(
        ctx: *mut McCtx,
        dst: *mut c_void,
        src: *const c_void,
        bytes: usize,
    ) -> c_int;
    pub fn mc_set_trace(ctx: *mut McCtx, buf: *mut u64, n: c_int) -> c_int;
    pub fn mc_set_wait_limit(ctx: *mut McCtx, ns: u64) -> c_int;
    pub fn mc_set_test_flags(ctx: *mut McCtx, flags: c_int) -> c_int;
    pub fn mc_eval_math(ctx: *mut McCtx, op: c_int, x: *const f32, y: *mut f32, n: c_int) -> c_int;
}

/// The library's error for a nonzero return code, with its message.
#[derive(Debug)]
pub struct McError {
    pub code: c_int,
    pub message: String,
}

pub fn check(rc: c_int) -> Result<(), McError> {
    if rc == MC_OK {
        return Ok(());
    }
    let msg = unsafe { CStr::from_ptr(mc_last_error()) }.to_string_lossy().into_owned();
    Err(McError { code: rc, message: msg })
}
