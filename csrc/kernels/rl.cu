// rl.cu — the per-sample RL math of the PPO trainer (sm_100a).
//
//   * surf_sample_heads: one warp per env samples every action head from the
//     policy output row: discrete heads by Gumbel-max over their logits, the
//     optional continuous yaw head from N(mu, exp(log_std)); writes the env's
//     action row (int32 x 8, shipped to the host as is) and the summed log-prob.
//     Reference: HeadPacker/sample_padded, python/train_fast.py:404-426.
//   * surf_gae: generalized advantage estimation, one thread per env scanning
//     the T decisions backwards in registers (reference: a 128-iteration
//     Python loop of tensor ops, python/train_fast.py:2119-2133).
//   * surf_train_pool: the rows the update samples from (train stride, ez-greedy
//     burst rows left out);
//   * surf_adv_moments: per-minibatch sum / sum of squares of the advantages
//     (double) for a whole epoch's permutation, so normalisation statistics
//     can be reduced across ranks before the loss runs.
//   * surf_ppo_loss: clipped-surrogate PPO loss, value loss and entropy bonus
//     for a minibatch, with its gradient w.r.t. the policy logits and value
//     computed in closed form in the same kernel (reference: mb_step's
//     log_softmax / entropy / ratio / clip chain + autograd,
//     python/train_fast.py:1846-1864).
//
// Random numbers: Philox-4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random
// numbers: as easy as 1, 2, 3", SC 2011), keyed by (seed, stream) and counted
// by (env, decision), so a decision's actions do not depend on the launch.
#include <cstdint>
#include <type_traits>

#include "surf_cuda.cuh"

namespace {

constexpr int kMaxHeads = 8;

struct HeadSpec {
  int n_heads;                 // discrete heads
  int size[kMaxHeads];         // categories per head
  int offset[kMaxHeads];       // first logit column of the head
  int slot[kMaxHeads];         // action-row slot the head drives
  int cont;                    // 1: column `cont_col` holds the yaw mean
  int cont_col;
  int width;                   // logits row length
  int neutral[6];              // value of sim slots no head drives
};

// ez-greedy temporally-extended exploration (reference: --ez-eps / --ez-mu /
// --ez-max, python/train_fast.py:748-761, 1952-1971): with probability eps per
// decision an env that runs no burst starts one: a uniformly random category
// for every discrete head, held for n ~ floor(u^(-1/(mu-1))) decisions
// (u uniform, a zeta-like heavy tail) clamped to [1, max_len]. While a burst
// runs, its action row replaces the sampled one and the decision is flagged
// off-policy (the update leaves flagged rows out of its sample pool).
struct EzArgs {
  float eps;          // 0: off
  float inv_mu1;      // 1 / (mu - 1)
  int max_len;
  int* left;          // [n] decisions left in the env's burst (persistent)
  int32_t* act;       // [n, 8] the burst's action row (persistent)
  uint8_t* flag;      // [n] out: 1 = burst action this decision
};

// ---- Philox-4x32-10 --------------------------------------------------------
struct U4 { uint32_t x, y, z, w; };
__device__ __forceinline__ U4 philox(U4 c, uint32_t k0, uint32_t k1) {
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(0xD2511F53u, c.x), lo0 = 0xD2511F53u * c.x;
    const uint32_t hi1 = __umulhi(0xCD9E8D57u, c.z), lo1 = 0xCD9E8D57u * c.z;
    c = U4{hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c;
}
// uniform in (0, 1): 24 random bits, centred in their bin
__device__ __forceinline__ float u01(uint32_t x) { return (static_cast<float>(x >> 8) + 0.5f) * (1.0f / 16777216.0f); }

template <typename T> __device__ __forceinline__ float ld(const T* p);
template <> __device__ __forceinline__ float ld<float>(const float* p) { return *p; }
template <> __device__ __forceinline__ float ld<uint16_t>(const uint16_t* p) { return surfk::bf16_to_f32(*p); }

__device__ __forceinline__ float warp_max(float v) {
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---- sampling ----------------------------------------------------------------
template <typename T>
__global__ void sample_kernel(const T* logits, int64_t ld_logits, HeadSpec hs, const float* log_std, int n,
                              uint64_t seed, uint64_t counter0, const int64_t* counter_ptr, int greedy, int32_t* act,
                              int64_t ld_act, float* logp_out, float* value_src, int64_t ld_value, float* value_out,
                              const uint8_t* fail_src, EzArgs ez) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= n) return;
  // decision counter: a device value (advanced by the trainer, so captured
  // graphs draw fresh noise on every replay) plus this launch's offset
  const uint64_t counter = counter0 + (counter_ptr ? static_cast<uint64_t>(*counter_ptr) : 0ull);
  const T* row = logits + warp * ld_logits;
  int32_t* out = act + warp * ld_act;
  float logp = 0.0f;
  const uint32_t k0 = static_cast<uint32_t>(seed), k1 = static_cast<uint32_t>(seed >> 32);
  for (int h = 0; h < hs.n_heads; ++h) {
    const int sz = hs.size[h];
    // lane j holds category j (heads have <= 32 categories)
    const float z = lane < sz ? ld<T>(row + hs.offset[h] + lane) : -INFINITY;
    const float m = warp_max(z);
    const float lse = m + logf(warp_sum(lane < sz ? expf(z - m) : 0.0f));
    float key = z;
    if (!greedy) {
      U4 r = philox(U4{static_cast<uint32_t>(warp), static_cast<uint32_t>(h * 32 + lane),
                       static_cast<uint32_t>(counter), static_cast<uint32_t>(counter >> 32)}, k0, k1);
      key = z - logf(-logf(u01(r.x)));          // Gumbel-max
    }
    if (lane >= sz) key = -INFINITY;
    // argmax with lowest index on ties
    float best = key;
    int bi = lane;
    for (int o = 16; o; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
    const float za = __shfl_sync(0xffffffffu, z, bi);
    logp += za - lse;
    if (lane == 0) out[hs.slot[h]] = bi;
  }
  if (lane == 0) {
    for (int s = 0; s < 6; ++s)
      if (hs.neutral[s] >= 0) out[s] = hs.neutral[s];
    if (hs.cont) {
      const float mu = ld<T>(row + hs.cont_col);
      const float ls = *log_std;
      float a = mu;
      if (!greedy) {
        U4 r = philox(U4{static_cast<uint32_t>(warp), 0xFFFFu, static_cast<uint32_t>(counter),
                         static_cast<uint32_t>(counter >> 32)}, k0 ^ 0x5bd1e995u, k1);
        const float u1 = u01(r.x), u2 = u01(r.y);
        const float g = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);   // Box-Muller
        a = mu + expf(ls) * g;
      }
      const float zz = (a - mu) * expf(-ls);
      logp += -0.5f * zz * zz - ls - 0.91893853320467274f;           // log sqrt(2 pi)
      out[6] = __float_as_int(a);
    } else {
      out[6] = 0;
    }
    out[7] = fail_src ? fail_src[warp] : 0;     // stall kill for the env's next step
    if (logp_out) logp_out[warp] = logp;
    if (value_out) value_out[warp] = value_src[warp * ld_value];
    if (ez.eps > 0.0f) {
      int left = ez.left[warp];
      int32_t* row_ez = ez.act + warp * 8;
      if (left == 0) {
        const U4 r = philox(U4{static_cast<uint32_t>(warp), 0xE2E2u, static_cast<uint32_t>(counter),
                               static_cast<uint32_t>(counter >> 32)}, k0 ^ 0x27D4EB2Fu, k1 ^ 0x165667B1u);
        if (u01(r.x) < ez.eps) {
          const float u = fmaxf(u01(r.y), 1e-6f);
          const int len = static_cast<int>(powf(u, -ez.inv_mu1));
          left = len < 1 ? 1 : (len > ez.max_len ? ez.max_len : len);
          for (int s = 0; s < 6; ++s) row_ez[s] = hs.neutral[s] >= 0 ? hs.neutral[s] : 0;
          for (int h0 = 0; h0 < hs.n_heads; h0 += 4) {
            const U4 q = philox(U4{static_cast<uint32_t>(warp), 0xE3E3u + static_cast<uint32_t>(h0),
                                   static_cast<uint32_t>(counter), static_cast<uint32_t>(counter >> 32)},
                                k0 ^ 0x27D4EB2Fu, k1 ^ 0x165667B1u);
            const uint32_t words[4] = {q.x, q.y, q.z, q.w};
            for (int j = 0; j < 4 && h0 + j < hs.n_heads; ++j) {
              const int h = h0 + j, sz = hs.size[h];
              const int cat = static_cast<int>(u01(words[j]) * static_cast<float>(sz));
              row_ez[hs.slot[h]] = cat < sz ? cat : sz - 1;
            }
          }
        }
      }
      const bool live = left > 0;
      if (live) {
        for (int s = 0; s < 6; ++s) out[s] = row_ez[s];
        --left;
      }
      ez.left[warp] = left;
      ez.flag[warp] = live ? 1 : 0;
    }
  }
}

// ---- training pool ------------------------------------------------------------
// Rows r = t * n + e of a rollout that the update samples from: decisions
// t = offset, offset + stride, ... (reference --train-stride,
// python/train_fast.py:2162-2168) whose action was on-policy (ez flag 0,
// :2170-2177). One block: each thread compacts a contiguous run of rows, a
// block-wide scan places the runs, so the pool keeps row order.
__global__ void __launch_bounds__(1024) train_pool_kernel(const uint8_t* ez_flag, int T, int n, int stride,
                                                          int offset, int64_t* pool, int64_t* count) {
  const int64_t total = static_cast<int64_t>(T) * n;
  const int64_t per = (total + blockDim.x - 1) / blockDim.x;
  const int64_t lo = threadIdx.x * per, hi = min(total, lo + per);
  auto keep = [&](int64_t r) {
    const int t = static_cast<int>(r / n);
    if (t < offset || (t - offset) % stride) return false;
    return !(ez_flag && ez_flag[r]);
  };
  int64_t mine = 0;
  for (int64_t r = lo; r < hi; ++r) mine += keep(r) ? 1 : 0;
  __shared__ int64_t scan[1024];
  scan[threadIdx.x] = mine;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {           // Hillis-Steele inclusive scan
    const int64_t v = threadIdx.x >= o ? scan[threadIdx.x - o] : 0;
    __syncthreads();
    scan[threadIdx.x] += v;
    __syncthreads();
  }
  int64_t at = scan[threadIdx.x] - mine;
  for (int64_t r = lo; r < hi; ++r)
    if (keep(r)) pool[at++] = r;
  if (threadIdx.x == blockDim.x - 1) *count = scan[threadIdx.x];
}

// ---- GAE ---------------------------------------------------------------------
__global__ void gae_kernel(const float* rew, const float* val, const float* done, const float* last_val, int T, int n,
                           float gamma, float lam, float* adv, float* ret, double* moments) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  double s = 0.0, s2 = 0.0;
  if (i < n) {
    float next_v = last_val[i], next_a = 0.0f;
    for (int t = T - 1; t >= 0; --t) {
      const int64_t k = static_cast<int64_t>(t) * n + i;
      const float nonterm = 1.0f - done[k];
      const float v = val[k];
      const float delta = rew[k] + gamma * next_v * nonterm - v;
      next_a = delta + gamma * lam * nonterm * next_a;
      adv[k] = next_a;
      ret[k] = next_a + v;
      next_v = v;
      s += next_a;
      s2 += static_cast<double>(next_a) * next_a;
    }
  }
  if (moments) {
    for (int o = 16; o; o >>= 1) { s += __shfl_xor_sync(0xffffffffu, s, o); s2 += __shfl_xor_sync(0xffffffffu, s2, o); }
    if ((threadIdx.x & 31) == 0) { atomicAdd(moments, s); atomicAdd(moments + 1, s2); }
  }
}

// per-minibatch moments: block b of minibatch m sums adv[perm[m*mb + j]]
__global__ void adv_moments_kernel(const float* adv, const int64_t* perm, int64_t mb, int n_mb, double* out) {
  const int m = blockIdx.y;
  double s = 0.0, s2 = 0.0;
  for (int64_t j = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; j < mb;
       j += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float a = adv[perm[m * mb + j]];
    s += a;
    s2 += static_cast<double>(a) * a;
  }
  for (int o = 16; o; o >>= 1) { s += __shfl_xor_sync(0xffffffffu, s, o); s2 += __shfl_xor_sync(0xffffffffu, s2, o); }
  if ((threadIdx.x & 31) == 0) { atomicAdd(out + 2 * m, s); atomicAdd(out + 2 * m + 1, s2); }
}

// ---- PPO loss + gradient -------------------------------------------------------
struct LossArgs {
  const float* coef;    // device: clip range, value coefficient, entropy coefficient
  float count;          // samples the loss averages over (global minibatch size)
  int norm_adv;
  int64_t n_src;        // rows of act / old_logp / adv / ret (an idx outside is reported, the row skipped)
  int* err;             // device error flag (may be null)
};

// gradient store: fp32, or bf16 (the backward GEMMs' operand; rounded as
// a separate fp32 -> bf16 conversion would round it)
__device__ __forceinline__ void st_grad(float* p, float v) { *p = v; }
__device__ __forceinline__ void st_grad(uint16_t* p, float v) { *p = surfk::f32_to_bf16(v); }

// Reductions over a group of GW lanes (the group's lanes are contiguous).
template <int GW>
__device__ __forceinline__ float group_max(float v) {
  for (int o = GW / 2; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o, GW));
  return v;
}
template <int GW>
__device__ __forceinline__ float group_sum(float v) {
  for (int o = GW / 2; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o, GW);
  return v;
}

// stats[0..5]: policy loss, value loss, entropy, approx_kl, clip fraction, samples (sums)
// RW rows per warp, one group of GW = 32 / RW lanes each (RW = 2 when every
// head has at most 16 categories: half the instructions per row). Every lane
// runs every shuffle; rows past n or with an unreadable index compute on row
// 0 / source 0 and write zeros (bad) or nothing (past n).
template <typename T, typename G, int RW>
__global__ void ppo_loss_kernel(const T* logits, int64_t ld_logits, const float* value, int64_t ld_value,
                                const int32_t* act, int64_t ld_act, const float* old_logp, const float* adv,
                                const float* ret, const int64_t* idx, const double* moments, HeadSpec hs,
                                const float* log_std, LossArgs la, int n, G* dlogits, int64_t ld_dlogits,
                                G* dvalue, int64_t ld_dvalue, float* dlog_std, float* stats) {
  constexpr int GW = 32 / RW;
  const int lane = threadIdx.x & 31;
  const int gl = lane % GW;                                   // lane within the row's group
  const int r = static_cast<int>((blockIdx.x * blockDim.x + threadIdx.x) >> 5) * RW + lane / GW;
  const bool in = r < n;
  float pg = 0, vl = 0, ent = 0, kl = 0, clipped = 0, dls = 0;
  const float clip = la.coef[0], vf_coef = la.coef[1], ent_coef = la.coef[2];
  int64_t src = in ? (idx ? idx[r] : r) : 0;
  const bool bad = in && (src < 0 || src >= la.n_src);
  if (bad && gl == 0) surfk::report_error(la.err, surfk::kErrLossIndex);
  if (bad) {                        // no gradient from a row that cannot be read
    for (int c = gl; c < hs.width; c += GW) st_grad(dlogits + r * ld_dlogits + c, 0.0f);
    if (gl == 0) st_grad(dvalue + r * ld_dvalue, 0.0f);
  }
  const bool live = in && !bad;
  if (!live) src = 0;
  const int rr = in ? r : 0;
  {
    const T* row = logits + rr * ld_logits;
    const int32_t* a = act + src * ld_act;
    // pass 1: log-prob and entropy of every head
    float logp = 0.0f, H = 0.0f;
    float lse_h[kMaxHeads];
    for (int h = 0; h < hs.n_heads; ++h) {
      const int sz = hs.size[h];
      const float z = gl < sz ? ld<T>(row + hs.offset[h] + gl) : -INFINITY;
      const float m = group_max<GW>(z);
      const float e = gl < sz ? expf(z - m) : 0.0f;
      const float sum = group_sum<GW>(e);
      const float lse = m + logf(sum);
      lse_h[h] = lse;
      const float lp = z - lse;
      const float p = e / sum;
      H += -group_sum<GW>(gl < sz ? p * lp : 0.0f);
      logp += __shfl_sync(0xffffffffu, lp, a[hs.slot[h]], GW);
    }
    float mu = 0.0f, ls = 0.0f, za = 0.0f;
    if (hs.cont) {
      mu = ld<T>(row + hs.cont_col);
      ls = *log_std;
      za = (__int_as_float(a[6]) - mu) * expf(-ls);
      logp += -0.5f * za * za - ls - 0.91893853320467274f;
      H += 0.5f + 0.91893853320467274f + ls;
    }
    float A = adv[src];
    if (la.norm_adv) {
      const double mean = moments[0] / la.count;
      const double var = (moments[1] - la.count * mean * mean) / (la.count - 1.0);
      A = static_cast<float>((A - mean) / (sqrt(var > 0 ? var : 0.0) + 1e-8));
    }
    const float diff = logp - old_logp[src];
    const float ratio = expf(diff);
    const float lo = 1.0f - clip, hi = 1.0f + clip;
    const float rc = fminf(fmaxf(ratio, lo), hi);
    const float s1 = -A * ratio, s2 = -A * rc;
    pg = fmaxf(s1, s2);
    // d(policy loss)/d(logp): the unclipped branch is the active one
    const float g_logp = (s1 >= s2) ? -A * ratio / la.count : 0.0f;
    const float v = value[rr * ld_value];
    const float dv = v - ret[src];
    vl = 0.5f * dv * dv;
    ent = H;
    kl = -diff;
    clipped = fabsf(ratio - 1.0f) > clip ? 1.0f : 0.0f;
    // gradients w.r.t. the logits of each head:
    //   policy  g_logp * (onehot - p)
    //   entropy -ent_coef/B * dH/dz = ent_coef/B * p * (log p + H_head)
    const float ce = ent_coef / la.count;
    for (int h = 0; h < hs.n_heads; ++h) {
      const int sz = hs.size[h];
      const float z = gl < sz ? ld<T>(row + hs.offset[h] + gl) : 0.0f;
      const float lp = z - lse_h[h];
      const float p = gl < sz ? expf(lp) : 0.0f;
      const float Hh = -group_sum<GW>(gl < sz ? p * lp : 0.0f);
      if (live && gl < sz) {
        const float onehot = (gl == a[hs.slot[h]]) ? 1.0f : 0.0f;
        st_grad(dlogits + r * ld_dlogits + hs.offset[h] + gl, g_logp * (onehot - p) + ce * p * (lp + Hh));
      }
    }
    if (hs.cont && gl == 0) {
      // d logp/d mu = za/sigma ; d logp/d log_std = za^2 - 1 ; dH/d log_std = 1
      if (live) st_grad(dlogits + r * ld_dlogits + hs.cont_col, g_logp * za * expf(-ls));
      dls = g_logp * (za * za - 1.0f) - ce;
    }
    if (live && gl == 0) st_grad(dvalue + r * ld_dvalue, vf_coef * dv / la.count);
  }
  // block reduction of the statistics, one atomic per block and field
  __shared__ float red[16][8];
  const int grp = threadIdx.x / GW;                           // < 8 * RW
  if (gl == 0) {
    red[grp][0] = live ? pg : 0.f;
    red[grp][1] = live ? vl : 0.f;
    red[grp][2] = live ? ent : 0.f;
    red[grp][3] = live ? kl : 0.f;
    red[grp][4] = live ? clipped : 0.f;
    red[grp][5] = live ? 1.f : 0.f;
    red[grp][6] = live ? dls : 0.f;
  }
  __syncthreads();
  if (threadIdx.x < 7) {
    float acc = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x / GW); ++w) acc += red[w][threadIdx.x];
    if (threadIdx.x < 6) atomicAdd(stats + threadIdx.x, acc);
    else if (hs.cont) atomicAdd(dlog_std, acc);
  }
}

HeadSpec make_spec(const int* sizes, int n_heads, const int* slots, int cont, const int* neutral) {
  HeadSpec hs{};
  hs.n_heads = n_heads;
  int off = 0;
  for (int h = 0; h < n_heads && h < kMaxHeads; ++h) {
    hs.size[h] = sizes[h];
    hs.offset[h] = off;
    hs.slot[h] = slots[h];
    off += sizes[h];
  }
  hs.cont = cont;
  hs.cont_col = off;
  hs.width = off + (cont ? 1 : 0);
  for (int s = 0; s < 6; ++s) hs.neutral[s] = neutral[s];
  return hs;
}

}  // namespace

// Head spec: n_heads discrete heads of `sizes` categories driving action-row
// slots `slots`; cont != 0 adds a continuous yaw mean column after them.
// neutral[6]: value for each sim slot no head drives (-1 = a head drives it).
SURF_EXPORT int surf_sample_heads(const void* logits, int logits_bf16, int64_t ld_logits, const int* sizes, int n_heads,
                                  const int* slots, int cont, const int* neutral, const float* log_std, int n,
                                  uint64_t seed, uint64_t counter, const int64_t* counter_ptr, int greedy,
                                  int32_t* act, int64_t ld_act,
                                  float* logp, const float* value_src, int64_t ld_value, float* value_out,
                                  const uint8_t* fail_src, const EzArgs* ez_in, void* stream) {
  if (n_heads > kMaxHeads) return static_cast<int>(cudaErrorInvalidValue);
  EzArgs ez{};
  if (ez_in && ez_in->eps > 0.0f) {
    if (!ez_in->left || !ez_in->act || !ez_in->flag || ez_in->max_len < 1) return static_cast<int>(cudaErrorInvalidValue);
    ez = *ez_in;
  }
  for (int h = 0; h < n_heads; ++h)
    if (sizes[h] > 32) return static_cast<int>(cudaErrorInvalidValue);
  HeadSpec hs = make_spec(sizes, n_heads, slots, cont, neutral);
  const int threads = 256, blocks = static_cast<int>(surfk::ceil_div(static_cast<int64_t>(n) * 32, threads));
  auto s = static_cast<cudaStream_t>(stream);
  if (logits_bf16)
    sample_kernel<uint16_t><<<blocks, threads, 0, s>>>(static_cast<const uint16_t*>(logits), ld_logits, hs, log_std, n,
                                                       seed, counter, counter_ptr, greedy, act, ld_act, logp,
                                                       const_cast<float*>(value_src), ld_value, value_out, fail_src,
                                                       ez);
  else
    sample_kernel<float><<<blocks, threads, 0, s>>>(static_cast<const float*>(logits), ld_logits, hs, log_std, n, seed,
                                                    counter, counter_ptr, greedy, act, ld_act, logp,
                                                    const_cast<float*>(value_src),
                                                    ld_value, value_out, fail_src, ez);
  SURF_RETURN_LAUNCH();
}

SURF_EXPORT int surf_gae(const float* rew, const float* val, const float* done, const float* last_val, int T, int n,
                         float gamma, float lam, float* adv, float* ret, double* moments, void* stream) {
  gae_kernel<<<static_cast<int>(surfk::ceil_div(n, 128)), 128, 0, static_cast<cudaStream_t>(stream)>>>(
      rew, val, done, last_val, T, n, gamma, lam, adv, ret, moments);
  SURF_RETURN_LAUNCH();
}

// out: double [n_mb, 2] (accumulated; zero it first)
SURF_EXPORT int surf_adv_moments(const float* adv, const int64_t* perm, int64_t mb, int n_mb, double* out, void* stream) {
  dim3 grid(static_cast<unsigned>(surfk::ceil_div(mb, 256 * 8) > 0 ? surfk::ceil_div(mb, 256 * 8) : 1), n_mb);
  adv_moments_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(adv, perm, mb, n_mb, out);
  SURF_RETURN_LAUNCH();
}

// dout_bf16: dlogits / dvalue are bf16 (the backward's operand) instead of fp32.
SURF_EXPORT int surf_ppo_loss(const void* logits, int logits_bf16, int64_t ld_logits, const float* value,
                              int64_t ld_value, const int32_t* act, int64_t ld_act, const float* old_logp,
                              const float* adv, const float* ret, const int64_t* idx, const double* moments,
                              const int* sizes, int n_heads, const int* slots, int cont, const float* log_std,
                              const float* coef, float count, int norm_adv, int n,
                              void* dlogits, int64_t ld_dlogits, void* dvalue, int64_t ld_dvalue, int dout_bf16,
                              float* dlog_std, float* stats, int64_t n_src, int* err, void* stream) {
  const int neutral[6] = {-1, -1, -1, -1, -1, -1};
  HeadSpec hs = make_spec(sizes, n_heads, slots, cont, neutral);
  LossArgs la{coef, count, norm_adv, n_src, err};
  bool narrow = true;                      // every head fits a 16-lane group: two rows per warp
  for (int h = 0; h < n_heads; ++h) narrow = narrow && sizes[h] <= 16;
  const int rw = narrow ? 2 : 1;
  const int threads = 256;
  const int blocks = static_cast<int>(surfk::ceil_div(surfk::ceil_div(static_cast<int64_t>(n), rw) * 32, threads));
  auto s = static_cast<cudaStream_t>(stream);
  auto run = [&](auto* dl, auto* dv) {
    using DL = std::remove_pointer_t<decltype(dl)>;
    if (logits_bf16) {
      auto* lg = static_cast<const uint16_t*>(logits);
      if (narrow)
        ppo_loss_kernel<uint16_t, DL, 2><<<blocks, threads, 0, s>>>(lg, ld_logits, value, ld_value, act, ld_act, old_logp,
                                                                    adv, ret, idx, moments, hs, log_std, la, n, dl,
                                                                    ld_dlogits, dv, ld_dvalue, dlog_std, stats);
      else
        ppo_loss_kernel<uint16_t, DL, 1><<<blocks, threads, 0, s>>>(lg, ld_logits, value, ld_value, act, ld_act, old_logp,
                                                                    adv, ret, idx, moments, hs, log_std, la, n, dl,
                                                                    ld_dlogits, dv, ld_dvalue, dlog_std, stats);
    } else {
      auto* lg = static_cast<const float*>(logits);
      if (narrow)
        ppo_loss_kernel<float, DL, 2><<<blocks, threads, 0, s>>>(lg, ld_logits, value, ld_value, act, ld_act, old_logp,
                                                                 adv, ret, idx, moments, hs, log_std, la, n, dl,
                                                                 ld_dlogits, dv, ld_dvalue, dlog_std, stats);
      else
        ppo_loss_kernel<float, DL, 1><<<blocks, threads, 0, s>>>(lg, ld_logits, value, ld_value, act, ld_act, old_logp,
                                                                 adv, ret, idx, moments, hs, log_std, la, n, dl,
                                                                 ld_dlogits, dv, ld_dvalue, dlog_std, stats);
    }
  };
  if (dout_bf16) run(static_cast<uint16_t*>(dlogits), static_cast<uint16_t*>(dvalue));
  else run(static_cast<float*>(dlogits), static_cast<float*>(dvalue));
  SURF_RETURN_LAUNCH();
}

// pool: int64 [T * n] (the first *count entries are written); count: one int64.
SURF_EXPORT int surf_train_pool(const uint8_t* ez_flag, int T, int n, int stride, int offset, int64_t* pool,
                                int64_t* count, void* stream) {
  if (T < 1 || n < 1 || stride < 1 || offset < 0 || offset >= stride) return static_cast<int>(cudaErrorInvalidValue);
  train_pool_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(ez_flag, T, n, stride, offset, pool, count);
  SURF_RETURN_LAUNCH();
}

__global__ void counter_add_kernel(int64_t* c, int64_t inc) { *c += inc; }

// *counter += inc (stream-ordered; used to advance the sampling counter once per rollout)
SURF_EXPORT int surf_counter_add(int64_t* counter, int64_t inc, void* stream) {
  counter_add_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(counter, inc);
  SURF_RETURN_LAUNCH();
}
