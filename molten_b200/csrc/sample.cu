// Sampling draw on the logits (the temperature > 0 token step): repetition penalty,
// temperature, top-k, top-p and the Gumbel-max draw, all on the device, the
// token folded into the same 64-bit key the greedy head writes so the token
// tail (mc_token_tail) serves both paths. Contract of the reference
// (docs/PROTOCOL.md:48-75, lfm_sample.metal:1-27, lfm/sample.rs:248-338):
//
//   w_i = pen(v_i) / T (v_i the f32 value of the bf16 logit; pen divides a
//         positive logit of a seen token by the penalty, multiplies a
//         non-positive one by it);
//   kept set {w >= tau}: top-k keeps every token whose w is at least the
//         k-th largest (ties kept); top-p then keeps the smallest set of most
//         likely tokens (among those) whose probability reaches top_p, a tie
//         group at the boundary kept whole; at least one token is kept;
//   draw: the kept token with the largest w + G_i, G_i a Gumbel(0, 1)
//         variate from word id % 4 of Philox4x32-10 with counter (id / 4,
//         pos, "SAMP", 0) and key (seed mod 2^32, seed / 2^32); ties to the
//         lower id.
//
// B200 design. The threshold tau is found by radix selection on the 32-bit
// orderable key of w, three digits (11, 11, 10 bits) per selection, with
// every sum an integer: top-k counts tokens, top-p sums per-token masses
// m_i = rint(exp(w_i - max w) * 2^40) (this project's fixed point; exp is
// mc_exp), so Z and every partial mass are exact 64-bit integers and the
// result does not depend on how the vocabulary is split over CTAs or on the
// order of any atomic. The top-p target is ceil(top_p_fix * Z / 2^32) with
// top_p_fix = rint(top_p * 2^32), in 128-bit integer arithmetic. One level
// is one launch over the vocabulary (2048 tokens per CTA, a shared-memory
// histogram of 2048 bins, its non-zero bins added to a global one); the CTA
// that finishes last (an atomic count, nothing waits) scans the bins from the
// top, keeps the digit whose cumulative total first reaches the target and
// clears the histogram for the next level.
//
// Launches: temperature only -> one (draw); top-k or top-p -> prep, three
// levels, draw; both -> prep, six levels, draw. The workspace's control part
// (plan and histogram) is zero before the first call and every call leaves
// it zero; the processed logits after it are scratch.
#include "mc_internal.cuh"

namespace {

constexpr int kTG = 256;          // threads of the wide kernels
constexpr int kTokPerThread = 4;  // prep / draw: 1024 tokens per CTA
constexpr int kLvTok = 2048;      // level kernels: tokens per CTA (8 per thread)
constexpr int kBins = 2048;
constexpr int kShift[3] = {21, 10, 0};
constexpr int kBits[3] = {11, 11, 10};
constexpr float kFix = 1099511627776.0f;  // 2^40

struct Params {
  const uint16_t* logits;
  const uint32_t* seen;  // bitmap or null
  float inv_temp, penalty, inv_penalty;
  uint32_t top_k;        // 0 = off
  uint64_t p_fix;        // rint(top_p * 2^32); 2^32 = off
  uint32_t seed_lo, seed_hi, pos;
  const uint32_t* pos_dev;  // when set, the position is read here (device feedback)
  int vocab;
  unsigned long long* key;
};

__device__ __forceinline__ uint32_t draw_pos(const Params& P) {
  return P.pos_dev ? *P.pos_dev : P.pos;
}

// Workspace: the plan, the global histogram, then w[vocab].
struct Plan {
  uint32_t mkey;     // orderable key of max w (prep, atomic max)
  uint32_t done;     // CTAs finished in the current launch
  uint32_t prefix;   // key bits resolved so far
  uint32_t tau_k;    // top-k threshold key
  uint32_t tau;      // final threshold key
  uint32_t pad[3];
  unsigned long long need;   // target still to reach inside the prefix
  unsigned long long above;  // mass of the keys above the prefix (top-k pass)
  unsigned long long zk;     // mass of the keys >= tau_k
  unsigned long long pad2;
};
static_assert(sizeof(Plan) == 64, "plan layout");

constexpr size_t kPlanBytes = 256;
constexpr size_t kHistBytes = (size_t)kBins * (4 + 8);

struct WsView {
  Plan* plan;
  uint32_t* hcnt;
  unsigned long long* hmass;
  float* w;
};

__host__ __device__ inline WsView ws_view(void* ws) {
  uint8_t* b = static_cast<uint8_t*>(ws);
  WsView v;
  v.plan = reinterpret_cast<Plan*>(b);
  v.hcnt = reinterpret_cast<uint32_t*>(b + kPlanBytes);
  v.hmass = reinterpret_cast<unsigned long long*>(b + kPlanBytes + 4 * kBins);
  v.w = reinterpret_cast<float*>(b + kPlanBytes + kHistBytes);
  return v;
}

__device__ __forceinline__ bool seen_bit(const uint32_t* seen, int i) {
  return seen && ((seen[i >> 5] >> (i & 31)) & 1u);
}

__device__ __forceinline__ unsigned long long token_mass(float w, float M) {
  const float e = mc_exp(__fsub_rn(w, M));
  if (!(e == e)) return 0ull;
  return __float2ull_rn(__fmul_rn(e, kFix));
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long k) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) {
    const unsigned long long o = __shfl_xor_sync(0xffffffffu, k, m);
    k = o > k ? o : k;
  }
  return k;
}

// Folds the CTA's best key into *key (one atomic per CTA).
__device__ __forceinline__ void cta_fold_key(unsigned long long k, unsigned long long* key) {
  __shared__ unsigned long long part[kTG / 32];
  k = warp_max_u64(k);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = k;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long b = part[0];
    for (int s = 1; s < kTG / 32; ++s) b = part[s] > b ? part[s] : b;
    if (b) atomicMax(key, b);
  }
}

// Pass 1: w for every token, and its max (as a key).
__global__ void __launch_bounds__(kTG) sample_prep_kernel(const Params P, void* ws) {
  mc_pdl_launch_dependents();
  mc_pdl_wait();
  const WsView V = ws_view(ws);
  const int i0 = (blockIdx.x * kTG + threadIdx.x) * kTokPerThread;
  uint32_t kmax = 0u;
  if (i0 < P.vocab) {
    const uint2 raw = *reinterpret_cast<const uint2*>(P.logits + i0);
    const uint16_t h[4] = {(uint16_t)raw.x, (uint16_t)(raw.x >> 16), (uint16_t)raw.y,
                           (uint16_t)(raw.y >> 16)};
    float4 w;
    float* wp = &w.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      wp[j] = mc_sample_w(mc_bf16_to_f32(h[j]), seen_bit(P.seen, i0 + j), P.inv_temp, P.penalty,
                          P.inv_penalty);
      const uint32_t k = mc_fkey(wp[j]);
      kmax = k > kmax ? k : kmax;
    }
    *reinterpret_cast<float4*>(V.w + i0) = w;
  }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) {
    const uint32_t o = __shfl_xor_sync(0xffffffffu, kmax, m);
    kmax = o > kmax ? o : kmax;
  }
  __shared__ uint32_t part[kTG / 32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = kmax;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t b = part[0];
    for (int s = 1; s < kTG / 32; ++s) b = part[s] > b ? part[s] : b;
    atomicMax(&V.plan->mkey, b);
  }
}

// ceil(p_fix * z / 2^32) in 128-bit arithmetic, at least 1.
__device__ __forceinline__ unsigned long long top_p_target(unsigned long long p_fix,
                                                           unsigned long long z) {
  const unsigned long long lo = p_fix * z, hi = __umul64hi(p_fix, z);
  // (hi:lo + 2^32 - 1) >> 32
  const unsigned long long lo2 = lo + 0xffffffffull;
  const unsigned long long hi2 = hi + (lo2 < lo ? 1ull : 0ull);
  const unsigned long long t = (hi2 << 32) | (lo2 >> 32);
  return t ? t : 1ull;
}

// One radix level. MASS 0: count selection (top-k; the masses are summed too,
// for Z_k); MASS 1: mass selection (top-p).
template <int MASS, int LEVEL>
__global__ void __launch_bounds__(kTG) sample_level_kernel(const Params P, void* ws) {
  mc_pdl_launch_dependents();
  mc_pdl_wait();
  const WsView V = ws_view(ws);
  __shared__ uint32_t scnt[kBins];
  __shared__ unsigned long long smass[kBins];
  __shared__ unsigned long long tsum[kTG], tmass[kTG];
  __shared__ uint32_t is_last;
  const int t = threadIdx.x;
  for (int b = t; b < kBins; b += kTG) {
    scnt[b] = 0u;
    smass[b] = 0ull;
  }
  const float M = mc_kfloat(V.plan->mkey);
  const uint32_t prefix = V.plan->prefix;
  const int shift = kShift[LEVEL], hb = kShift[LEVEL] + kBits[LEVEL];
  const uint32_t mask = (1u << kBits[LEVEL]) - 1u;
  __syncthreads();
  const int base = blockIdx.x * kLvTok;
  for (int j = 0; j < kLvTok / kTG; ++j) {
    const int i = base + j * kTG + t;
    if (i >= P.vocab) break;
    const float w = V.w[i];
    const uint32_t k = mc_fkey(w);
    if (LEVEL > 0 && (k >> hb) != (prefix >> hb)) continue;
    const uint32_t bin = (k >> shift) & mask;
    atomicAdd(&scnt[bin], 1u);
    atomicAdd(&smass[bin], token_mass(w, M));
  }
  __syncthreads();
  for (int b = t; b < kBins; b += kTG) {
    if (scnt[b]) {
      atomicAdd(V.hcnt + b, scnt[b]);
      atomicAdd(V.hmass + b, smass[b]);
    }
  }
  __threadfence();
  __syncthreads();
  if (t == 0) {
    const uint32_t done = atomicAdd(&V.plan->done, 1u);
    is_last = done == gridDim.x - 1 ? 1u : 0u;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // ---- the last CTA: bins from the top, thread t owns bins
  // [kBins - 8(t + 1), kBins - 8t) in decreasing order
  Plan* pl = V.plan;
  unsigned long long need;
  if (LEVEL == 0) {
    if (MASS == 0) {
      need = P.top_k;
    } else {
      unsigned long long z = 0ull;
      if (P.top_k) {
        z = pl->zk;
      } else {  // Z over the whole vocabulary: every token is in a level-0 bin
        unsigned long long zt = 0ull;
        for (int b = t; b < kBins; b += kTG) zt += __ldcg(V.hmass + b);
        tmass[t] = zt;
        __syncthreads();
        for (int s = 0; s < kTG; ++s) z += tmass[s];
        __syncthreads();
      }
      need = top_p_target(P.p_fix, z);
    }
  } else {
    need = pl->need;
  }
  unsigned long long vals[8], ms[8];
  unsigned long long own = 0ull, ownm = 0ull;
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const int b = kBins - 1 - (8 * t + r);
    const unsigned long long c = __ldcg(V.hcnt + b);
    const unsigned long long m = __ldcg(V.hmass + b);
    ms[r] = m;
    vals[r] = MASS ? m : c;
    own += vals[r];
    ownm += m;
  }
  tsum[t] = own;
  tmass[t] = ownm;
  __syncthreads();
  // exclusive prefix from the top (sequential over 256 partials: exact integers)
  unsigned long long before = 0ull, beforem = 0ull;
  for (int s = 0; s < t; ++s) {
    before += tsum[s];
    beforem += tmass[s];
  }
  __shared__ int found_t;
  if (t == 0) found_t = -1;
  __syncthreads();
  if (before < need && before + own >= need) found_t = t;
  __syncthreads();
  if (found_t < 0 && t == 0) {
    // rounding cannot leave the total short of the target (counts: top_k <
    // vocab; masses: the target is at most Z); keep everything as a guard
    found_t = -2;
  }
  __syncthreads();
  if (t == (found_t >= 0 ? found_t : kTG - 1)) {
    int d = 7;
    unsigned long long cum = before, cumm = beforem;
    if (found_t >= 0) {
      for (int r = 0; r < 8; ++r) {
        if (cum + vals[r] >= need) {
          d = r;
          break;
        }
        cum += vals[r];
        cumm += ms[r];
      }
    } else {
      for (int r = 0; r < 7; ++r) {
        cum += vals[r];
        cumm += ms[r];
      }
    }
    const uint32_t digit = (uint32_t)(kBins - 1 - (8 * t + d)) & mask;
    const uint32_t pre = (LEVEL == 0 ? 0u : pl->prefix) | (digit << shift);
    const unsigned long long rest = need > cum ? need - cum : 1ull;
    if (MASS == 0) {
      const unsigned long long above = (LEVEL == 0 ? 0ull : pl->above) + cumm;
      if (LEVEL == 2) {
        pl->tau_k = pre;
        pl->zk = above + ms[d];
        pl->prefix = 0u;
        pl->need = 0ull;
        pl->above = 0ull;
        pl->tau = pre;  // final unless a top-p pass follows
      } else {
        pl->prefix = pre;
        pl->need = rest;
        pl->above = above;
      }
    } else {
      if (LEVEL == 2) {
        pl->tau = pre;
        pl->prefix = 0u;
        pl->need = 0ull;
      } else {
        pl->prefix = pre;
        pl->need = rest;
      }
    }
  }
  // clear the histogram for the next level, and the completion count
  for (int b = t; b < kBins; b += kTG) {
    V.hcnt[b] = 0u;
    V.hmass[b] = 0ull;
  }
  if (t == 0) pl->done = 0u;
}

// The draw: the kept token (w >= tau; FULL: every token, w computed here)
// with the largest w + G folded into the key; the last CTA clears the plan.
template <int FULL>
__global__ void __launch_bounds__(kTG) sample_draw_kernel(const Params P, void* ws) {
  mc_pdl_launch_dependents();
  mc_pdl_wait();
  const int i0 = (blockIdx.x * kTG + threadIdx.x) * kTokPerThread;
  unsigned long long best = 0ull;
  if (FULL) {
    if (i0 < P.vocab) {
      const uint2 raw = *reinterpret_cast<const uint2*>(P.logits + i0);
      const uint16_t h[4] = {(uint16_t)raw.x, (uint16_t)(raw.x >> 16), (uint16_t)raw.y,
                             (uint16_t)(raw.y >> 16)};
      uint32_t c[4] = {(uint32_t)i0 >> 2, draw_pos(P), MC_SAMPLE_DOMAIN, 0u};
      mc_philox4x32_10(c, P.seed_lo, P.seed_hi);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float w = mc_sample_w(mc_bf16_to_f32(h[j]), seen_bit(P.seen, i0 + j), P.inv_temp,
                                    P.penalty, P.inv_penalty);
        const unsigned long long k = mc_argmax_key(__fadd_rn(w, mc_gumbel(c[j])), i0 + j);
        best = k > best ? k : best;
      }
    }
    cta_fold_key(best, P.key);
    return;
  }
  const WsView V = ws_view(ws);
  const uint32_t tau = V.plan->tau;
  if (i0 < P.vocab) {
    const float4 w4 = *reinterpret_cast<const float4*>(V.w + i0);
    const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
    bool any = false;
#pragma unroll
    for (int j = 0; j < 4; ++j) any |= mc_fkey(wv[j]) >= tau;
    if (any) {
      uint32_t c[4] = {(uint32_t)i0 >> 2, draw_pos(P), MC_SAMPLE_DOMAIN, 0u};
      mc_philox4x32_10(c, P.seed_lo, P.seed_hi);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (mc_fkey(wv[j]) < tau) continue;
        const unsigned long long k = mc_argmax_key(__fadd_rn(wv[j], mc_gumbel(c[j])), i0 + j);
        best = k > best ? k : best;
      }
    }
  }
  cta_fold_key(best, P.key);
  __shared__ uint32_t is_last;
  __threadfence();
  if (threadIdx.x == 0) is_last = atomicAdd(&V.plan->done, 1u) == gridDim.x - 1 ? 1u : 0u;
  __syncthreads();
  if (is_last && threadIdx.x == 0) {
    Plan* pl = V.plan;
    pl->mkey = 0u;
    pl->tau_k = 0u;
    pl->tau = 0u;
    pl->zk = 0ull;
    pl->done = 0u;
  }
}

__global__ void sample_mark_kernel(const uint32_t* tok, uint32_t* seen, int vocab,
                                   uint32_t* pos_dev) {
  mc_pdl_launch_dependents();
  mc_pdl_wait();
  if (threadIdx.x == 0) {
    const uint32_t t = *tok;
    if (seen && t < (uint32_t)vocab) seen[t >> 5] |= 1u << (t & 31u);
    if (pos_dev) *pos_dev += 1u;
  }
}

template <typename K>
int launch(K kernel, int grid, const Params& P, void* ws, mc_ctx* ctx, const char* what) {
  MC_CUDA(mc_launch_pdl(kernel, dim3(grid), dim3(kTG), 0, ctx->stream, P, ws));
  return mc_after_launch(what);
}

}  // namespace

extern "C" size_t mc_sample_workspace_bytes(int vocab) {
  return kPlanBytes + kHistBytes + 4 * (size_t)(vocab > 0 ? vocab : 0);
}

extern "C" int mc_sample_draw(mc_ctx* ctx, const uint16_t* logits, int vocab, const uint32_t* seen,
                              const mc_sampling* s, uint32_t pos, const uint32_t* pos_dev,
                              unsigned long long* key, void* workspace, size_t ws_bytes) {
  MC_REQUIRE(ctx, "sample_draw: null context");
  MC_REQUIRE(s, "sample_draw: null sampling parameters");
  MC_REQUIRE(logits && key, "sample_draw: null logits or key");
  MC_REQUIRE(vocab >= 4 && vocab % 4 == 0 && vocab <= (1 << 24),
             "sample_draw: vocab %d must be a multiple of 4 in [4, 2^24]", vocab);
  MC_REQUIRE(s->temperature >= 1e-6f && s->temperature == s->temperature &&
                 s->temperature <= 3.0e38f,
             "sample_draw: temperature must be >= 1e-6 (0 = greedy, not drawn)");
  MC_REQUIRE(s->top_p > 0.0f && s->top_p <= 1.0f, "sample_draw: top_p must be in (0, 1]");
  MC_REQUIRE(s->repetition_penalty >= 1e-6f && s->repetition_penalty <= 1e6f,
             "sample_draw: repetition_penalty must be in [1e-6, 1e6]");
  const bool penalty = s->repetition_penalty != 1.0f;
  MC_REQUIRE(!penalty || seen, "sample_draw: a repetition penalty needs the seen set");
  MC_REQUIRE(mc_aligned(logits, 8) && mc_aligned(key, 8),
             "sample_draw: logits and key must be 8-byte aligned");
  const uint32_t top_k = s->top_k >= (uint32_t)vocab ? 0u : s->top_k;  // k >= vocab is off
  const bool use_p = s->top_p < 1.0f;
  const bool full = top_k == 0 && !use_p;
  if (!full) {
    MC_REQUIRE(workspace && mc_aligned(workspace, 256), "sample_draw: workspace must be 256-byte aligned");
    MC_REQUIRE(ws_bytes >= mc_sample_workspace_bytes(vocab),
               "sample_draw: workspace of %zu bytes < %zu", ws_bytes,
               mc_sample_workspace_bytes(vocab));
  }
  Params P;
  P.logits = logits;
  P.seen = penalty ? seen : nullptr;
  P.inv_temp = 1.0f / s->temperature;
  P.penalty = s->repetition_penalty;
  P.inv_penalty = 1.0f / s->repetition_penalty;
  P.top_k = top_k;
  // rint(top_p * 2^32): exact scaling, then round to nearest
  P.p_fix = (uint64_t)llrintf(s->top_p * 4294967296.0f);
  P.seed_lo = (uint32_t)s->seed;
  P.seed_hi = (uint32_t)(s->seed >> 32);
  P.pos = pos;
  P.pos_dev = pos_dev;
  P.vocab = vocab;
  P.key = key;
  const int wide = (vocab + kTG * kTokPerThread - 1) / (kTG * kTokPerThread);
  if (full) return launch(sample_draw_kernel<1>, wide, P, workspace, ctx, "sample_draw_kernel");
  const int lv = (vocab + kLvTok - 1) / kLvTok;
  int rc;
  if ((rc = launch(sample_prep_kernel, wide, P, workspace, ctx, "sample_prep_kernel"))) return rc;
  if (top_k) {
    if ((rc = launch(sample_level_kernel<0, 0>, lv, P, workspace, ctx, "sample_level_kernel")) ||
        (rc = launch(sample_level_kernel<0, 1>, lv, P, workspace, ctx, "sample_level_kernel")) ||
        (rc = launch(sample_level_kernel<0, 2>, lv, P, workspace, ctx, "sample_level_kernel")))
      return rc;
  }
  if (use_p) {
    if ((rc = launch(sample_level_kernel<1, 0>, lv, P, workspace, ctx, "sample_level_kernel")) ||
        (rc = launch(sample_level_kernel<1, 1>, lv, P, workspace, ctx, "sample_level_kernel")) ||
        (rc = launch(sample_level_kernel<1, 2>, lv, P, workspace, ctx, "sample_level_kernel")))
      return rc;
  }
  return launch(sample_draw_kernel<0>, wide, P, workspace, ctx, "sample_draw_kernel");
}

extern "C" int mc_sample_mark(mc_ctx* ctx, const uint32_t* tok, uint32_t* seen, int vocab,
                              uint32_t* pos_dev) {
  MC_REQUIRE(ctx, "sample_mark: null context");
  MC_REQUIRE(tok && (seen || pos_dev) && vocab >= 1, "sample_mark: bad arguments");
  MC_CUDA(mc_launch_pdl(sample_mark_kernel, dim3(1), dim3(32), 0, ctx->stream, tok, seen, vocab,
                        pos_dev));
  return mc_after_launch("sample_mark_kernel");
}
