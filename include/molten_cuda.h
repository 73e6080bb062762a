/*
 * molten_cuda.h -- C ABI of the B200 (sm_100a) quantized MoE matmul path.
 *
 * Drop-in boundary for the op-level surface that Molten's
 * src/kernels/{lfm,quant,elementwise}.rs expose to src/lfm.rs. Every entry
 * point below names the reference function it replaces (paths inside the
 * reference project). A Rust `src/cuda.rs` binds these with `extern "C"`
 * declarations mirroring the prototypes below; tests and bench.py bind them
 * with ctypes.
 *
 * Conventions
 *  - All pointers are DEVICE pointers owned by the caller (mc_copy_async
 *    also takes page-locked host pointers); no compute entry point
 *    allocates device memory (scratch is passed in, as the reference's
 *    `Scratch` is preallocated by the caller, lfm.rs:557-626) -- except
 *    mc_ep_alloc (expert-parallel exchange buffers); the scratch of
 *    mc_moe_decode_layer_noalloc is a static device array of the library.
 *  - bf16 values travel as uint16_t bit patterns.
 *  - Work is enqueued on the context's stream and is asynchronous, like
 *    `ComputePass::dispatch_at` (metal.rs:326-355); mc_sync is `commit_wait`.
 *  - Return 0 on success or a negative MC_E* code; the message is in
 *    mc_last_error() (thread-local). Argument checks run before anything is
 *    enqueued, so a rejected call leaves nothing half-issued, like the
 *    reference's `ensure!`s before encoding (quant.rs:42-66).
 *  - One context per thread and device; calls are not re-entrant.
 *  - Q4 = MLX affine 4-bit, group 64: codes u32[out][in/8], low nibble first;
 *    Q6 = 4 codes per 3 bytes (little-endian 6-bit stream), codes u32 words
 *    [out][in*6/32]; scales/biases bf16[out][in/64]; w = s*q + b
 *    (weights.rs:7-20).
 */
#ifndef MOLTEN_CUDA_H
#define MOLTEN_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MC_OK 0
#define MC_EINVAL (-1)       /* bad shape, dtype, alignment or pointer */
#define MC_ECUDA (-2)        /* CUDA runtime error */
#define MC_EUNSUPPORTED (-3) /* shape this build does not instantiate */
#define MC_ENCCL (-4)        /* NCCL error (expert parallelism) */
#define MC_ETIMEOUT (-5)     /* a bounded wait ran out */

#define MC_ROUTE_SOFTMAX_RENORM 0 /* BASELINE: softmax over E, top-4, renormalise */
#define MC_ROUTE_SIGMOID_BIAS 1   /* reference model: sigmoid + expert_bias selection */

#define MC_DTYPE_BF16 0
#define MC_DTYPE_F32 1

typedef struct mc_ctx mc_ctx;

/* QuantWeights (weights.rs:11-30). Device pointers, caller-owned. */
typedef struct mc_qweights {
  const uint32_t* codes;
  const uint16_t* scales;
  const uint16_t* biases;
  int32_t out_features;
  int32_t in_features;
  int32_t group_size;
  int32_t bits;
} mc_qweights;

/* ---------------------------------------------------------------- context */

/* MetalContext::new (metal.rs:91-147): binds `device`; `stream` is the
 * cudaStream_t to enqueue on (NULL = the default stream). */
int mc_create(int device, void* stream, mc_ctx** out);
int mc_destroy(mc_ctx* ctx);
/* Switches the stream later calls enqueue on (NULL = the default stream). */
int mc_set_stream(mc_ctx* ctx, void* stream);
/* ComputePass::commit_wait (metal.rs:383-399): waits for all enqueued work
 * and reports any asynchronous CUDA error. */
int mc_sync(mc_ctx* ctx);
const char* mc_last_error(void);
/* Library build id, e.g. "molten_cuda sm_100a". */
const char* mc_version(void);

/* check_quant (quant.rs:42-66): validates a weight descriptor without a GPU
 * call. Returns 0 or MC_EINVAL with the reason in mc_last_error(). */
int mc_check_quant(const mc_qweights* w);

/* ------------------------------------------------------------ decode path */

/* gemv_quant (kernels/lfm.rs:112-149 -> lfm_gemv_q4_bf16_k2048
 * lfm.metal:161-183, lfm_gemv_q6_bf16_x4 :245-297): y[b] = W . x[b] for
 * `batch` independent bf16 rows x[batch][in] -> y[batch][out]. bits 4 or 6,
 * in <= 4096; 4-bit rows also up to in = 16384 (lfm_gemv_q4_bf16_k11776,
 * the dense FFN's down projection). */
int mc_gemv_quant(mc_ctx* ctx, const mc_qweights* w, const uint16_t* x, uint16_t* y,
                  int batch);

/* gemv_head_argmax (kernels/lfm.rs:826-844 -> lfm_gemv_q6_bf16_x4_argmax
 * lfm.metal:1215-1282): fused head GEMV + argmax over bf16-rounded logits,
 * folded into keys[b] by 64-bit atomic max. keys[batch] must be zero on entry
 * (mc_token_tail clears them). */
int mc_gemv_head_argmax(mc_ctx* ctx, const mc_qweights* w, const uint16_t* x,
                        unsigned long long* keys, int batch);

/* token_tail (kernels/lfm.rs:850-888 -> lfm_token_tail lfm.metal:1291-1386):
 * reads and clears keys[b], writes out_tok[b]; when `embed` is non-NULL also
 * writes the next input row x_next[b] = embed[tok] (bf16 table [vocab][hidden])
 * and its RMSNorm normed_next[b] with gain norm_w. */
int mc_token_tail(mc_ctx* ctx, unsigned long long* keys, uint32_t* out_tok,
                  const uint16_t* embed, int vocab, const uint16_t* norm_w,
                  uint16_t* x_next, uint16_t* normed_next, int hidden, float eps,
                  int batch);

/* argmax_bf16 (kernels/lfm.rs:794-820 -> lfm.metal:1126-1192): argmax over
 * stored bf16 logits[batch][n], ties to the lowest index. */
int mc_argmax_bf16(mc_ctx* ctx, const uint16_t* logits, int n, uint32_t* out, int batch);

/* add_rmsnorm_bf16 (norm.metal:63-136, via lfm_norm_row_v8_tg
 * lfm.metal:306-366): hout = bf16(h + b) (b may be NULL), nout =
 * RMSNorm(hout) * w. hidden = 2048. */
int mc_add_rmsnorm(mc_ctx* ctx, const uint16_t* h, const uint16_t* b, const uint16_t* w,
                   uint16_t* hout, uint16_t* nout, int hidden, float eps, int batch);

/* router_addnorm_route (kernels/lfm.rs:266-311 -> lfm_router_addnorm_route_f32
 * lfm.metal:773-854): residual add + RMSNorm + router GEMV + top-4 in one
 * launch. router_w is [E][hidden] in router_dtype (MC_DTYPE_BF16 for the
 * BASELINE router, MC_DTYPE_F32 for the reference model's). expert_bias
 * (f32[E], nullable) is used by MC_ROUTE_SIGMOID_BIAS. counter: u32[batch]
 * zeroed words the kernel leaves zeroed. E = 64, hidden = 2048. */
int mc_router_addnorm_route(mc_ctx* ctx, const uint16_t* h, const uint16_t* b,
                            const uint16_t* norm_w, uint16_t* h_out, uint16_t* normed,
                            const void* router_w, int router_dtype, const float* expert_bias,
                            int route_mode, float* logits, uint32_t* ids, uint16_t* weights,
                            uint32_t* counter, int n_experts, int hidden, float eps,
                            float route_eps, int batch);

/* gemv_f32 (kernels/lfm.rs:314-335 -> lfm.metal:417-428): unfused router
 * logits[batch][E] = W . x[batch] (prompt-final row). */
int mc_gemv_router(mc_ctx* ctx, const void* router_w, int router_dtype, const uint16_t* x,
                   float* logits, int n_experts, int hidden, int batch);

/* route_token (kernels/lfm.rs:391-417 -> lfm_route_warp_f32 lfm.metal:686-703):
 * top-4 ids and bf16 weights from logits[batch][E]. */
int mc_route_token(mc_ctx* ctx, const float* logits, int n_experts, int route_mode,
                   const float* expert_bias, float route_eps, uint32_t* ids,
                   uint16_t* weights, int batch);

/* gemv_gather_act (kernels/lfm.rs:421-460 -> lfm_gemv_q4_gather_act_bf16
 * lfm.metal:1392-1445): act[b][r][i] = silu(gate row)*up row for the four
 * selected experts ids[b][r]; gate/up stacked [E*I][H] Q4. */
int mc_gemv_gather_act(mc_ctx* ctx, const mc_qweights* gate, const mc_qweights* up,
                       const uint16_t* x, const uint32_t* ids, uint16_t* act, int n_experts,
                       int batch);

/* gemv_gather_down_combine4 (kernels/lfm.rs:499-533 ->
 * lfm_gemv_q4_gather_down_combine4_bf16 lfm.metal:1503-1554): down GEMVs of
 * the four selected experts (stacked [E*H][I] Q4) with the weighted combine. */
int mc_gemv_gather_down_combine4(mc_ctx* ctx, const mc_qweights* down, const uint16_t* act,
                                 const uint32_t* ids, const uint16_t* weights, uint16_t* out,
                                 int n_experts, int batch);

/* moe_decode (lfm.rs:967-1011) behind the fused router (lfm.rs:1154-1169):
 * one persistent launch does router_addnorm_route + gemv_gather_act +
 * gemv_gather_down_combine4 for ONE token (batch 1), bit-identical to the
 * three separate calls. `workspace` holds mc_moe_decode_workspace_words(I)
 * u32 words, zeroed once before the first call and then owned by one chain
 * of calls (it keeps an epoch and tagged intermediate values between calls;
 * workspace[2] != 0 after a call reports a bounded wait that gave up (1) or
 * an expert id out of range (2); the act rows are the bf16 values
 * ((uint16_t*)(workspace + 136))[r*I + i]). All row buffers, the weights'
 * scales/biases and the workspace 16-byte aligned; the expert width I is a
 * multiple of 64 and at most 2048. */
size_t mc_moe_decode_workspace_words(int moe_inter);
int mc_moe_decode_layer(mc_ctx* ctx, const uint16_t* h, const uint16_t* b,
                        const uint16_t* norm_w, uint16_t* h_out, uint16_t* normed,
                        const void* router_w, int router_dtype, const float* expert_bias,
                        int route_mode, float* logits, uint32_t* ids, uint16_t* weights,
                        const mc_qweights* gate, const mc_qweights* up,
                        const mc_qweights* down, int n_experts, uint16_t* out,
                        uint32_t* workspace, size_t ws_words, float eps, float route_eps);

/* mc_moe_decode_layer with no workspace argument and no allocation: the
 * scratch is a fixed 33,312-byte array inside this library (one per device),
 * for callers that cannot lend device memory (an engine whose allocator is
 * frozen after start-up, a plugin barred from allocating on the serving
 * path). It has no counterpart in the reference, whose Metal kernels take
 * every buffer from the caller. Limits and duties:
 *  - expert width I = gate->out_features / n_experts at most 2048, else
 *    MC_EINVAL before any launch;
 *  - every argument is checked before anything is enqueued; then the
 *    array's address is looked up with ctx's device current, and the first
 *    call on each device also zeroes it on ctx's stream, waiting for that, so
 *    the first call blocks and must come before any stream capture; each
 *    call is then one kernel launch;
 *  - the scratch is shared by every context and stream of the process on a
 *    device, so calls whose kernels could overlap race: order them;
 *  - `status` (device u32, may be NULL) receives this call's status word,
 *    the codes mc_moe_decode_layer leaves in workspace[2]; the kernel clears
 *    the word in the array, so each call reports its own launch only;
 *  - a device reset (cudaDeviceReset) reloads the library's device code:
 *    the array then starts zeroed again, as on first use. */
int mc_moe_decode_layer_noalloc(mc_ctx* ctx, const uint16_t* h, const uint16_t* b,
                                const uint16_t* norm_w, uint16_t* h_out, uint16_t* normed,
                                const void* router_w, int router_dtype,
                                const float* expert_bias, int route_mode, float* logits,
                                uint32_t* ids, uint16_t* weights, const mc_qweights* gate,
                                const mc_qweights* up, const mc_qweights* down, int n_experts,
                                uint16_t* out, uint32_t* status, float eps, float route_eps);

/* gemv_quant(proj, h) -> b (kernels/lfm.rs:112-149) followed by
 * mc_moe_decode_layer(h, b, ...) in ONE launch: every CTA computes its slice
 * of b = bf16(proj . h) (proj: Q4 2048 x 2048, group 64) in the canonical
 * GEMV order, the slices are exchanged as epoch-tagged words and the layer
 * proceeds as mc_moe_decode_layer, so every output is bit-identical to the
 * two calls. The pairing is the decode step of BASELINE cfg4 (a Q4
 * projection of the layer input feeding the MoE layer's residual add); the
 * reference issues the two ops separately, and the saving is the kernel
 * boundary between them. `workspace` holds mc_moe_decode_proj_workspace_words(I)
 * words (mc_moe_decode_workspace_words(I) + 2048; b's tagged words follow
 * the act words); `p_out` (may be NULL) receives b; status bit 32 in
 * workspace[2] reports a projection wait that gave up. Other rules as
 * mc_moe_decode_layer. */
size_t mc_moe_decode_proj_workspace_words(int moe_inter);
int mc_moe_decode_layer_proj(mc_ctx* ctx, const uint16_t* h, const mc_qweights* proj,
                             uint16_t* p_out, const uint16_t* norm_w, uint16_t* h_out,
                             uint16_t* normed, const void* router_w, int router_dtype,
                             const float* expert_bias, int route_mode, float* logits,
                             uint32_t* ids, uint16_t* weights, const mc_qweights* gate,
                             const mc_qweights* up, const mc_qweights* down, int n_experts,
                             uint16_t* out, uint32_t* workspace, size_t ws_words, float eps,
                             float route_eps);

/* ------------------------------------------------ decode neighbours */

/* proj3_gemv_scatter (kernels/lfm.rs:150-205 -> lfm_proj3_gemv_scatter_bf16
 * lfm.metal:1020-1068): the Q, K and V Q4 GEMVs of one bf16 row x[2048] in
 * one launch: q_out[nq], k_out[nk], and V row i stored straight into the KV
 * cache at position pos: v_cache[((i / 64) * max_seq + pos) * 64 + i % 64]
 * (v_cache bf16 [nv / 64][max_seq][64]; no other cache entry is written). */
int mc_proj3_gemv_scatter(mc_ctx* ctx, const mc_qweights* q, const mc_qweights* k,
                          const mc_qweights* v, const uint16_t* x, uint16_t* q_out,
                          uint16_t* k_out, uint16_t* v_cache, int max_seq, int pos);

/* conv3_gemv (kernels/lfm.rs:207-246 -> lfm_conv3_gemv_split_bf16
 * lfm.metal:1070-1110): the short conv's input projection w_proj [3C][2048]
 * (rows c, C + c, 2C + c are channel c's b, c and x) on one bf16 row x, then
 * the two-tap conv with taps bf16 [C][3] and state bf16 [2][C]:
 * v2 = bf16(b * x), z = bf16((t0 * state[0][c] + t1 * state[1][c]) + t2 * v2),
 * out[c] = bf16(c * z), new_state[0][c] = state[1][c], new_state[1][c] = v2
 * (new_state must not alias state). */
int mc_conv3_gemv(mc_ctx* ctx, const mc_qweights* w_proj, const uint16_t* x,
                  const uint16_t* taps, const uint16_t* state, uint16_t* out,
                  uint16_t* new_state, int channels);

/* gemv_gu_act (kernels/lfm.rs:462-495 -> lfm_gemv_q4_gu_act_bf16
 * lfm.metal:1447-1498): the dense FFN front half, act[b][n] =
 * bf16(bf16(silu(bf16(gate_n . x[b]))) * bf16(up_n . x[b])) for bf16 rows
 * x[batch][in] (in <= 4096), act[batch][out]. */
int mc_gemv_gu_act(mc_ctx* ctx, const mc_qweights* gate, const mc_qweights* up,
                   const uint16_t* x, uint16_t* act, int batch);

/* ------------------------------------------------- sampling draw */

/* Sampling (lfm/sample.rs:87-213; docs/PROTOCOL.md:48-75): temperature
 * (>= 1e-6; temperature 0 is the greedy head, not this call), top_k (0 or
 * >= vocab: off), top_p in (0, 1] (1: off), repetition_penalty in
 * [1e-6, 1e6] (1: off), 64-bit seed. */
typedef struct mc_sampling {
  float temperature;
  uint32_t top_k;
  float top_p;
  float repetition_penalty;
  uint64_t seed;
} mc_sampling;

/* SampleScratch::encode_draw (lfm/sample.rs:248-338 -> lfm_sample_gumbel /
 * _prep / _levels / _gather / _finish, lfm_sample.metal:161-930): draws the
 * token at absolute position `pos` from the bf16 logits row [vocab] (vocab a
 * multiple of 4) into *key, the zeroed 64-bit argmax key the greedy head
 * writes, so mc_token_tail reads and clears it for both paths. w_i =
 * pen(v_i) / T; kept set {w >= tau} (top-k ties kept, then the smallest
 * top-p prefix with its boundary tie group); the kept token with the
 * largest w + Gumbel(Philox4x32-10 word) wins, ties to the lower id. `seen`
 * (u32 bitmap [vocab / 32], needed only with a penalty) marks the
 * sequence's tokens. The top-k / top-p threshold is exact: integer counts
 * and per-token masses rint(exp(w - max w) * 2^40) summed in 64 bits.
 * workspace: mc_sample_workspace_bytes(vocab) device bytes, 256-byte
 * aligned, zeroed once before the first call (every call leaves its control
 * words zero again; the rest is scratch); unused (may be NULL) when top_k
 * and top_p are both off. */
size_t mc_sample_workspace_bytes(int vocab);
/* pos_dev (nullable): read the position from this device word instead of
 * `pos`, so a decode step captured once in a CUDA graph draws each replay at
 * the next position (mc_sample_mark advances it). */
int mc_sample_draw(mc_ctx* ctx, const uint16_t* logits, int vocab, const uint32_t* seen,
                   const mc_sampling* s, uint32_t pos, const uint32_t* pos_dev,
                   unsigned long long* key, void* workspace, size_t ws_bytes);
/* SampleScratch::encode_mark (lfm/sample.rs:340-353 -> lfm_sample_mark
 * lfm_sample.metal:922-931): after mc_token_tail wrote *tok, sets its bit in
 * `seen` (nullable: no penalty) and, when pos_dev is set, advances the
 * device position by one. */
int mc_sample_mark(mc_ctx* ctx, const uint32_t* tok, uint32_t* seen, int vocab,
                   uint32_t* pos_dev);

/* ----------------------------------------------------------- prefill path */

/* moe_route_batch (kernels/lfm.rs:536-555 -> lfm.metal:1558-1602): per-token
 * top-4 ids[m][4] and bf16 gate weights gw[m][4] from logits[m][E]. */
int mc_moe_route_batch(mc_ctx* ctx, const float* logits, int m, int n_experts,
                       int route_mode, const float* expert_bias, float route_eps,
                       uint32_t* ids, uint16_t* gw);

/* moe_zero_counts .. moe_blocks (kernels/lfm.rs:557-697 -> lfm.metal:1604-1770)
 * in two launches: counts[E], offsets[E] (exclusive scan), the stable
 * token-major, rank-major scatter ids_sorted[m*4] / slotpos[m*4], and the
 * row-tile list tiles[max_tiles] of uint4 {m0, m_end, expert, 0} with its
 * length in *n_tiles (device u32): every full bm-row tile first, in expert
 * order, then the partial tiles by decreasing height (ties: lower expert).
 * bm is the tile height (256 for the grouped GEMMs, at most 256 there);
 * max_tiles >= ceil(m*4/bm) + E. */
int mc_moe_sort_map(mc_ctx* ctx, const uint32_t* ids, int m, int n_experts, int bm,
                    uint32_t* counts, uint32_t* offsets, uint32_t* ids_sorted,
                    uint32_t* slotpos, uint32_t* tiles, uint32_t* n_tiles, int max_tiles);

/* gather_rows_bf16 (elementwise.rs:59-104 -> elementwise.metal:41-52):
 * out[i] = table[ids[i]] for bf16 rows of width hidden. */
int mc_gather_rows_bf16(mc_ctx* ctx, const uint16_t* table, const uint32_t* ids, int rows,
                        int hidden, uint16_t* out);

/* Dense Q4 GEMM for the prefill's non-expert projections (replaces
 * dequant_q4_bf16_bulk + gemm_bf16_nt, quant.metal:69-114, gemm.rs:33-60, as
 * lfm.rs:661-671 calls them): c[m][N] = a[m][K] . bf16(s*q + b)[N][K]^T, the
 * weights dequantised on the fly into the tensor-core tiles (never written
 * out). Runs the grouped GEMM with one expert over 256-row chunks; the chunk
 * list goes to `workspace` (device, mc_gemm_q4_workspace_words(m) u32,
 * 16-byte aligned). N and K multiples of 128; status as for the grouped GEMM. */
size_t mc_gemm_q4_workspace_words(int m);
int mc_gemm_q4(mc_ctx* ctx, const uint16_t* a, int m, const mc_qweights* w, uint16_t* c,
               uint32_t* workspace, size_t ws_words, uint32_t* status);

/* gemm_q4_grouped_mlx (quant.rs:228-266 -> lfm_qmm_t_body
 * quant_nax.metal:4091-4234): C[i][n] = sum_k A[i][k] * bf16(s*q+b)[e*N+n][k]
 * for the rows i of each tile's expert e; A bf16 [rows][K] (expert-sorted),
 * C bf16 [rows][N]; w stacked [E*N][K] Q4; tiles/n_tiles from
 * mc_moe_sort_map with bm <= 256 (a tile taller than 256 rows is malformed).
 * tcgen05 tensor-core kernel (fp32 accumulation). status: nullable u32 word,
 * bit 0 = a bounded wait gave up, bit 1 = a malformed tile was skipped.
 * N % 128 == 0, K % 128 == 0. */
int mc_gemm_q4_grouped(mc_ctx* ctx, const uint16_t* a, int rows, const mc_qweights* w,
                       int n_experts, uint16_t* c, const uint32_t* tiles,
                       const uint32_t* n_tiles, int max_tiles, uint32_t* status);

/* gemm_q4_grouped_mlx_gu + silu_mul_bf16 (quant.rs:146-199,
 * elementwise.metal:7-15): the gate and up grouped GEMMs of a tile share the
 * A tile and the epilogue writes act = bf16(bf16(silu(g)) * u) with g, u the
 * bf16-rounded GEMM outputs. */
int mc_gemm_q4_grouped_gu(mc_ctx* ctx, const uint16_t* a, int rows, const mc_qweights* gate,
                          const mc_qweights* up, int n_experts, uint16_t* act,
                          const uint32_t* tiles, const uint32_t* n_tiles, int max_tiles,
                          uint32_t* status);

/* silu_mul_bf16 (elementwise.rs:48-56 -> elementwise.metal:7-15). */
int mc_silu_mul_bf16(mc_ctx* ctx, const uint16_t* gate, const uint16_t* up, uint16_t* out,
                     size_t n);

/* moe_combine_rows (kernels/lfm.rs:701-756 -> lfm_moe_combine_rows_bf16_v16
 * lfm.metal:915-940): out[t] = bf16(sum_r bf16(gw[t][r] * ed[slotpos[t][r]])). */
int mc_moe_combine_rows(mc_ctx* ctx, const uint16_t* ed, const uint32_t* slotpos,
                        const uint16_t* gw, uint16_t* out, int m, int topk, int hidden);

/* moe_prefill (lfm.rs:847-965) from router logits on: route, sort + tile
 * map, gather, grouped gate/up + SwiGLU, grouped down, combine (seven
 * launches, no host round trip). x bf16 [m][H], logits f32 [m][E]; gate/up
 * stacked [E*I][H], down [E*H][I] Q4; out bf16 [m][H]. workspace: device
 * bytes >= mc_moe_prefill_workspace_size(m, E, H, I), 256-byte aligned; it
 * holds the intermediates (ids, gate weights, sorted order, tiles, gx, act,
 * ed) and the GEMM status word. */
size_t mc_moe_prefill_workspace_size(int m, int n_experts, int hidden, int moe_inter);
int mc_moe_prefill(mc_ctx* ctx, const uint16_t* x, const float* logits, int m,
                   const mc_qweights* gate, const mc_qweights* up, const mc_qweights* down,
                   int n_experts, int route_mode, const float* expert_bias, void* workspace,
                   size_t ws_bytes, uint16_t* out);

/* ------------------------------------------- expert-parallel prefill (new)
 * No counterpart in the reference (its moe_prefill runs on one device). Rank
 * r of `world` holds experts [r*E/world, (r+1)*E/world); every rank sorted its
 * own pairs with mc_moe_sort_map and holds counts_all[world][E] (an
 * all-gather of every rank's counts). Receive buffers are expert-major (rows
 * of local expert j contiguous, sources in rank order); all ranks allocate
 * buffers of equal capacity. The caller puts a cross-rank barrier after
 * mc_ep_dispatch and after mc_ep_return (a receiver may read only once every
 * sender's copy finished). status (nullable u32) bit 2: rows beyond a
 * capacity were skipped (inconsistent counts). */

/* Relabels expert ids[n] in place through table[n_experts] (an expert
 * placement: model expert -> position in the rank-contiguous order). Ids out
 * of range stay and set status bit 1. */
int mc_map_ids(mc_ctx* ctx, uint32_t* ids, size_t n, const uint32_t* table, int n_experts,
               uint32_t* status);
/* Device memory whose base can be shared with other processes (cudaMalloc). */
int mc_ep_alloc(mc_ctx* ctx, size_t bytes, void** out);
int mc_ep_free(mc_ctx* ctx, void* ptr);
/* CUDA IPC: 64-byte handle of an mc_ep_alloc base; open / close a peer's. */
int mc_ipc_handle(mc_ctx* ctx, void* base, void* handle_out);
int mc_ipc_open(mc_ctx* ctx, const void* handle, void** out);
int mc_ipc_close(mc_ctx* ctx, void* ptr);
/* Copies this rank's expert-sorted rows x[ids_sorted[i]] (bf16 [m][hidden])
 * into the owners' receive buffers recv_bufs[world] (own and peer-mapped). */
int mc_ep_dispatch(mc_ctx* ctx, const uint16_t* x, int m, int hidden,
                   const uint32_t* ids_sorted, const uint32_t* counts_all, int rank, int world,
                   int n_experts, void* const* recv_bufs, size_t recv_cap_rows, uint32_t* status);
/* Row-chunk list (uint4 {m0, m_end, local expert, 0}, <= bm rows, full chunks
 * first then partial by decreasing height) of this rank's receive buffer,
 * its length in *n_tiles and the row count in *rows (nullable). */
int mc_ep_tiles(mc_ctx* ctx, const uint32_t* counts_all, int rank, int world, int n_experts,
                int bm, uint32_t* tiles, uint32_t* n_tiles, uint32_t* rows, int max_tiles);
/* Copies the expert outputs ed (bf16 [ed_rows][hidden], receive order) back to
 * the sources' slots in home_bufs[world] (their sorted order). */
int mc_ep_return(mc_ctx* ctx, const uint16_t* ed, size_t ed_rows, int hidden,
                 const uint32_t* counts_all, int rank, int world, int n_experts,
                 void* const* home_bufs, size_t home_cap_rows, uint32_t* status);

/* ------------------------- expert-parallel prefill through the C ABI alone
 * One process per GPU. A host with no PyTorch drives the whole step:
 *   rank 0: mc_ep_unique_id(id) and hands the 128 bytes to the other ranks
 *           (its own channel);
 *   every rank: mc_ep_init(ctx, W, rank, id, timeout_ms) -> a non-blocking
 *           NCCL communicator (set-up and teardown), every NCCL call watched
 *           with ncclCommGetAsyncError against the timeout and aborted past
 *           it;
 *           mc_ep_reserve(ctx, m_max, E, slots_per_rank, H, I) (collective:
 *           allocates the exchange buffers and maps every rank's through CUDA
 *           IPC);
 *           mc_ep_place(load, ...) on the same load matrix -> the same slot
 *           tables everywhere; the rank loads the weights of its slots
 *           (slot_expert[rank*spr ..]) stacked in slot order;
 *           mc_ep_moe_prefill(...) per step (collective; no host sync; the
 *           counts, token rows and expert rows move by peer stores between
 *           bounded device barriers);
 *           mc_ep_status(ctx, &st) when it wants the step's status bits
 *           (1 a GEMM wait, 2 a malformed tile or expert id, 4 rows beyond a
 *           capacity, 8 a cross-rank barrier that gave up); mc_sync waits for
 *           the stream while watching the communicator;
 *           mc_ep_finalize(ctx) (collective) at the end.
 * No counterpart in the reference, whose moe_prefill (lfm.rs:847-965) runs
 * on one device; the per-step arithmetic is moe_prefill's, so each rank's
 * output equals it within the grouped GEMMs' tolerance and its ids, sorted
 * order and slot positions are bit-exact. mc_ep_init and mc_ep_reserve
 * allocate (cudaMalloc) and synchronise; mc_ep_moe_prefill allocates
 * nothing. */
int mc_ep_unique_id(void* out128);
int mc_ep_init(mc_ctx* ctx, int nranks, int rank, const void* nccl_unique_id, int timeout_ms);
int mc_ep_reserve(mc_ctx* ctx, int m_max, int n_experts, int slots_per_rank, int hidden,
                  int moe_inter);
/* Host-only placement: load[s][e] (pairs of source rank s routed to expert
 * e, e.g. one routing pass) -> tables[s][e] (the slot source s sends expert
 * e's rows to) and slot_expert[W * slots_per_rank] (the expert each slot
 * holds, -1 if none). Spare slots (W * spr > E) replicate the hottest
 * experts. Deterministic. */
int mc_ep_place(const unsigned long long* load, int world, int n_experts, int slots_per_rank,
                uint32_t* tables, int32_t* slot_expert);
/* One step on this rank's m tokens (m <= m_max): x bf16 [m][H], logits f32
 * [m][E], the rank's slot weights gate/up [spr*I][H], down [spr*H][I],
 * slot_table (device u32 [E]: this rank's row of mc_ep_place's tables),
 * out bf16 [m][H]. */
int mc_ep_moe_prefill(mc_ctx* ctx, const uint16_t* x, const float* logits, int m,
                      const mc_qweights* gate, const mc_qweights* up, const mc_qweights* down,
                      const uint32_t* slot_table, int route_mode, const float* expert_bias,
                      uint16_t* out);
/* Waits for the stream; *out = the status bits since the last call (then
 * cleared). */
int mc_ep_status(mc_ctx* ctx, uint32_t* out);
/* The last step's pair counts of every rank [W][W * spr] (host copy; waits). */
int mc_ep_counts(mc_ctx* ctx, uint32_t* out, size_t n);
int mc_ep_finalize(mc_ctx* ctx);
/* Profiling aid: with `on`, each step records events at its phase
 * boundaries; mc_ep_phase_ms waits and writes the last step's seven phase
 * times in ms (route + relabel + sort, counts exchange + barrier, dispatch
 * with the row chunks and the return map, a slot kept for the barrier after
 * the dispatch -- its wait now runs inside the gate/up GEMM, so the slot is
 * ~0 --, grouped GEMMs + return, the barrier after them, combine). */
int mc_ep_set_profile(mc_ctx* ctx, int on);
int mc_ep_phase_ms(mc_ctx* ctx, float* out7);

/* Cross-layer prefetch hint (no reference counterpart): the next
 * mc_moe_decode_layer (or _noalloc) launched on ctx prefetches the byte
 * ranges [p0, p0 + n0) and [p1, p1 + n1) into L2 once its own expert rows are
 * streaming, and clears the setting. A decode loop passes the next layer's
 * router weights and RMSNorm weight, which every CTA of that layer waits for
 * first. NULL or 0 leaves a range out. */
int mc_set_l2_prefetch(mc_ctx* ctx, const void* p0, size_t n0, const void* p1, size_t n1);

/* Host <-> device staging (replaces Tensor::write_bytes, tensor.rs:127-146,
 * and the host reads of Tensor::contents / to_f32 / to_u32, tensor.rs:165-200,
 * which on the reference's unified memory touch the shared buffer directly).
 * Copies bytes from src to dst in ctx's stream order. When both are
 * addressable by the context's device -- its own memory, or page-locked host
 * memory mapped into the device address space -- and 16-byte aligned with a
 * size that is a multiple of 16, one small copy kernel does it (chained to
 * the kernels around it like the decode kernels, far shorter than a DMA copy
 * for the few-KB rows of a decode step); otherwise cudaMemcpyAsync. The
 * ranges must not overlap. Asynchronous: host memory read or written here
 * must stay untouched until the stream reaches the copy. */
int mc_copy_async(mc_ctx* ctx, void* dst, const void* src, size_t bytes);

/* -------------------------------------------------------------- test aid */

/* Profiling aid: when buf (device, n u64 words) is set, the persistent
 * kernels record %globaltimer at their phase boundaries, 16 words per CTA
 * (mc_moe_decode_layer: 0 start, 1 norm, 2 logits published, 3 top-4 known,
 * 13 copies issued, 8/9 first/last gate-up chunk landed, 4 gate/up done,
 * 5 act published, 10 act loaded, 11 down rows landed, 12 down computed,
 * 6 combine, 7 exit). NULL switches it off (the default). */
int mc_set_trace(mc_ctx* ctx, unsigned long long* buf, int n);

/* Limit of every bounded device wait (cross-CTA flags, copy barriers, peer
 * flags) of the kernels launched on ctx from now on, in nanoseconds; 0
 * restores each kernel's default (200 ms for the decode kernels, 1 s for the
 * grouped GEMMs and the expert-parallel barriers). A wait that runs out sets
 * the kernel's status bit and the kernel returns; nothing hangs. No
 * reference counterpart (Metal kernels there never wait on one another). */
int mc_set_wait_limit(mc_ctx* ctx, unsigned long long ns);

/* Test aid: flags that make later launches on ctx skip one step so that a
 * bounded wait runs out on purpose (the failure-detection tests use it with a
 * short mc_set_wait_limit). MC_TEST_SKIP_LOGIT_PUBLISH: the router warps of
 * mc_moe_decode_layer(_noalloc) publish no logits, so every CTA's logit wait
 * gives up and status bit 1 is set. 0 (the default) for normal work. */
#define MC_TEST_SKIP_LOGIT_PUBLISH 1
/* MC_TEST_SKIP_BARRIER_ARRIVE: the expert-parallel barrier of this rank
 * waits without arriving, so its wait runs out and sets status bit 8. */
#define MC_TEST_SKIP_BARRIER_ARRIVE 2
int mc_set_test_flags(mc_ctx* ctx, int flags);

/* Evaluates the library's device math on x[n] into y[n]: op 0 = mc_exp,
 * 1 = SiLU, 2 = sigmoid, 3 = bf16 rounding. Lets tests check the device
 * functions bit for bit against the CPU restatement. */
int mc_eval_math(mc_ctx* ctx, int op, const float* x, float* y, int n);

#ifdef __cplusplus
}
#endif
#endif /* MOLTEN_CUDA_H */
