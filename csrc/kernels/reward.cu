// reward.cu — per-decision reward shaping, observation features, curiosity
// counts and epoch permutations on the GPU (sm_100a).
//
// The env hands the GPU one record row per env and decision (pose, velocity,
// tick, summed base reward and done / trunc / goal / ended flags, see
// csrc/sim/env.hpp). surf_reward turns it into the training reward in one
// thread per env, keeping each env's reward state in device memory:
//
//   speed      (v_h - v_h,prev) * scale                    (reference SpeedReward)
//   avgspeed   v_h * scale                                  (AvgSpeedReward)
//   forward    new maxima of the spawn-yaw projection       (ForwardProgressReward)
//   path       horizontal distance, teleports filtered     (PathLengthReward)
//   maxspeed   new maxima of v_h                            (MaxSpeedReward)
//   coverage   v_h * scale on entering an unvisited cell of this episode,
//              -revisit_pen on re-entering one              (CoverageSpeedReward)
//   acro       coverage + style: banked air-spin rotation paid on landing a
//              real flight, switch (backwards) landings, backwards ramp
//              riding                                          (AcroCoverageReward)
//   blend      (1 - w) forward + w path, w annealed by the trainer (BlendedReward)
//   race       scale * (d_prev - d) - time_pen on the geodesic distance field
//              (trilinear over honest corners), success bonus (+ finish_k
//              time bonus), fail penalty, speed-equivalent potential with
//              its death refund, stagnation kill            (RaceReward)
// plus, for any mode, count-based curiosity int_coef / sqrt(N + 1) on moving
// into a new (cell x yaw sector x speed bin) key, counts hashed into a 2^k
// int32 table shared by all envs (two phases: bonuses from the counts before
// this decision, then the increments, as the reference's np.add.at does).
// Reference: python/surfgym/rewards.py:35-694. Rewards are evaluated once per
// decision of K ticks (the reference's per-decision mode): potential terms
// telescope exactly; the rest differ from per-tick sums by O(K) sampling.
#include <cstdint>

#include "surf_cuda.cuh"

namespace {

enum Mode : int { kSpeed = 0, kAvgSpeed = 1, kForward = 2, kPath = 3, kMaxSpeed = 4, kCoverage = 5, kRace = 6,
                  kAcro = 7, kBlend = 8 };
enum RecCol : int { kOx = 0, kOy = 1, kOz = 2, kYaw = 3, kVx = 6, kVy = 7, kVz = 8, kTick = 9, kBase = 10, kDone = 11,
                    kTrunc = 12, kGoal = 13, kEnded = 14, kOnground = 15 };

struct RewardParams {
  int mode, n, K;
  float scale, max_step, revisit_pen;
  // coverage cells
  float cmin[3], cell;
  int cdim[3];
  int cov_words;                  // uint32 words per env visited bitset
  // race
  const uint16_t* field;          // geodesic distance, uint16 * quant
  float quant, fmin[3], fcell, valid_max, sentinel;
  int fdim[3];
  float time_pen, success_bonus, finish_k, finish_tref, fail_pen, speed_coef, speed_equiv;
  int stall_ticks;
  float stall_eps;
  // curiosity
  float int_coef, int_cell;
  int int_view, int_speed;
  float int_min[3];
  int int_dim[3];
  uint32_t table_mask;            // table size - 1 (power of two)
  float gamma_boot;               // unused here (bootstraps are precomputed)
  // acro style terms (per tick; scaled by K per decision)
  float spin_bonus, switch_bonus, spin_rate_cap, back_bonus, gravity_tick;
  int max_spins, min_air;         // min_air in ticks
  // blend: weight w of path over forward, read from device memory (schedules
  // change it without re-capturing the graphs that launch this kernel)
  const float* blend_w;
};

// per-env state (float [n, kStateFloats])
constexpr int kStateFloats = 24;
enum St : int { sPx = 0, sPy = 1, sPz = 2, sSpeed = 3, sBest = 4, sSince = 5, sTicks = 6, sDirX = 7, sDirY = 8,
                sRefX = 9, sRefY = 10, sD = 11, sEpRet = 12, sEpLen = 13, sInit = 14, sCell = 15,
                sYaw = 16, sVx = 17, sVy = 18, sVz = 19, sStreak = 20, sSpin = 21, sBest2 = 22 };

__device__ __forceinline__ float wrap180(float a) {
  a = fmodf(a + 180.0f, 360.0f);
  if (a < 0.0f) a += 360.0f;
  return a - 180.0f;
}

__device__ __forceinline__ float hspeed(const float* r) { return sqrtf(r[kVx] * r[kVx] + r[kVy] * r[kVy]); }

// honest-corner trilinear sample of the goal field (uint16 distances * quant)
__device__ float field_sample(const RewardParams& p, float x, float y, float z) {
  const float gx = (x - p.fmin[0]) / p.fcell - 0.5f, gy = (y - p.fmin[1]) / p.fcell - 0.5f,
              gz = (z - p.fmin[2]) / p.fcell - 0.5f;
  const int i0 = static_cast<int>(floorf(gx)), j0 = static_cast<int>(floorf(gy)), k0 = static_cast<int>(floorf(gz));
  const float fx = gx - i0, fy = gy - j0, fz = gz - k0;
  float num = 0.0f, den = 0.0f;
  for (int dz = 0; dz < 2; ++dz)
    for (int dy = 0; dy < 2; ++dy)
      for (int dx = 0; dx < 2; ++dx) {
        const int ix = min(max(i0 + dx, 0), p.fdim[0] - 1);
        const int iy = min(max(j0 + dy, 0), p.fdim[1] - 1);
        const int iz = min(max(k0 + dz, 0), p.fdim[2] - 1);
        const float v = static_cast<float>(p.field[(static_cast<int64_t>(iz) * p.fdim[1] + iy) * p.fdim[0] + ix]) * p.quant;
        const float w = (dx ? fx : 1.0f - fx) * (dy ? fy : 1.0f - fy) * (dz ? fz : 1.0f - fz) * (v < p.valid_max ? 1.0f : 0.0f);
        num += w * v;
        den += w;
      }
  return den > 1e-6f ? num / den : p.sentinel;
}

__device__ __forceinline__ int64_t curiosity_key(const RewardParams& p, const float* r) {
  int c[3];
  const float pos[3] = {r[kOx], r[kOy], r[kOz]};
  for (int a = 0; a < 3; ++a) {
    int v = static_cast<int>(floorf((pos[a] - p.int_min[a]) / p.int_cell));
    c[a] = min(max(v, 0), p.int_dim[a] - 1);
  }
  int64_t key = c[0] + static_cast<int64_t>(p.int_dim[0]) * (c[1] + static_cast<int64_t>(p.int_dim[1]) * c[2]);
  if (p.int_view > 0) {
    float y = fmodf(r[kYaw], 360.0f);
    if (y < 0) y += 360.0f;
    const int yb = min(max(static_cast<int>(floorf(y / 360.0f * p.int_view)), 0), p.int_view - 1);
    key = key * p.int_view + yb;
  }
  if (p.int_speed > 0) {
    const int sb = min(max(static_cast<int>(hspeed(r) / (4000.0f / p.int_speed)), 0), p.int_speed - 1);
    key = key * p.int_speed + sb;
  }
  return key;
}

__device__ __forceinline__ uint32_t bucket(const RewardParams& p, int64_t key) {
  uint64_t z = static_cast<uint64_t>(key) + 0x9E3779B97F4A7C15ULL;     // SplitMix64 finaliser as the hash
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return static_cast<uint32_t>(z ^ (z >> 31)) & p.table_mask;
}

__device__ __forceinline__ int cov_cell(const RewardParams& p, const float* r) {
  int c[3];
  const float pos[3] = {r[kOx], r[kOy], r[kOz]};
  for (int a = 0; a < 3; ++a) {
    int v = static_cast<int>(floorf((pos[a] - p.cmin[a]) / p.cell));
    c[a] = min(max(v, 0), p.cdim[a] - 1);
  }
  return c[0] + p.cdim[0] * (c[1] + p.cdim[1] * c[2]);
}

// init: per-env state from the spawn records (first decision of a run)
__global__ void reward_init_kernel(RewardParams p, const float* rec, int64_t ld, float* st, uint32_t* visited,
                                   int64_t* keys) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= p.n) return;
  const float* r = rec + i * ld;
  float* s = st + static_cast<int64_t>(i) * kStateFloats;
  for (int k = 0; k < kStateFloats; ++k) s[k] = 0.0f;
  s[sPx] = r[kOx]; s[sPy] = r[kOy]; s[sPz] = r[kOz];
  s[sSpeed] = hspeed(r);
  s[sBest] = s[sSpeed];
  const float yaw = r[kYaw] * 0.017453292519943295f;
  s[sDirX] = cosf(yaw); s[sDirY] = sinf(yaw);
  s[sRefX] = r[kOx]; s[sRefY] = r[kOy];
  if (p.mode == kRace) { s[sD] = field_sample(p, r[kOx], r[kOy], r[kOz]); s[sBest] = s[sD]; }
  if (p.mode == kForward || p.mode == kBlend) s[sBest] = 0.0f;
  s[sYaw] = r[kYaw]; s[sVx] = r[kVx]; s[sVy] = r[kVy]; s[sVz] = r[kVz];
  if (p.mode == kCoverage || p.mode == kAcro) {
    uint32_t* v = visited + static_cast<int64_t>(i) * p.cov_words;
    for (int w = 0; w < p.cov_words; ++w) v[w] = 0;
    const int c = cov_cell(p, r);
    v[c >> 5] |= 1u << (c & 31);
    s[sCell] = __int_as_float(c);
  }
  if (p.int_coef > 0) keys[i] = curiosity_key(p, r);
  s[sInit] = 1.0f;
}

// phase 1: reward, state update, curiosity key; bonus read from current counts
__global__ void reward_kernel(RewardParams p, const float* rec, int64_t ld, float* st, uint32_t* visited,
                              const int* counts, float* boot, float* rew_out, float* done_out, uint8_t* stall,
                              int64_t* new_key, int64_t* keys, float* stats) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  float rr = 0.0f, ep_done = 0.0f, ep_ret = 0.0f, ep_len = 0.0f, succ = 0.0f, fail = 0.0f, trn = 0.0f, ibonus = 0.0f;
  if (i < p.n) {
    const float* r = rec + i * ld;
    float* s = st + static_cast<int64_t>(i) * kStateFloats;
    const bool ended = r[kEnded] != 0.0f, done = r[kDone] != 0.0f, goal = r[kGoal] != 0.0f;
    const float sp = hspeed(r);
    const float dx = r[kOx] - s[sPx], dy = r[kOy] - s[sPy];
    const float hstep = sqrtf(dx * dx + dy * dy);
    const bool teleported = hstep > p.max_step * p.K;
    switch (p.mode) {
      case kSpeed: rr = (sp - s[sSpeed]) * p.scale; break;
      case kAvgSpeed: rr = sp * p.scale; break;
      case kPath: rr = teleported ? 0.0f : hstep * p.scale; break;
      case kMaxSpeed:
        rr = fmaxf(sp - s[sBest], 0.0f) * p.scale;
        s[sBest] = fmaxf(s[sBest], sp);
        break;
      case kForward: {
        if (teleported) { s[sRefX] += dx; s[sRefY] += dy; }
        const float proj = (r[kOx] - s[sRefX]) * s[sDirX] + (r[kOy] - s[sRefY]) * s[sDirY];
        rr = fmaxf(proj - s[sBest], 0.0f) * p.scale;
        s[sBest] = fmaxf(s[sBest], proj);
        break;
      }
      case kBlend: {       // (1 - w) * forward + w * path, both anchors kept live
        if (teleported) { s[sRefX] += dx; s[sRefY] += dy; }
        const float proj = (r[kOx] - s[sRefX]) * s[sDirX] + (r[kOy] - s[sRefY]) * s[sDirY];
        const float fwd = fmaxf(proj - s[sBest], 0.0f) * p.scale;
        s[sBest] = fmaxf(s[sBest], proj);
        const float path = teleported ? 0.0f : hstep * p.scale;
        const float w = p.blend_w ? fminf(fmaxf(*p.blend_w, 0.0f), 1.0f) : 0.0f;
        rr = (1.0f - w) * fwd + w * path;
        break;
      }
      case kAcro:
      case kCoverage: {
        const int c = cov_cell(p, r);
        const int prev = __float_as_int(s[sCell]);
        uint32_t* v = visited + static_cast<int64_t>(i) * p.cov_words;
        if (c != prev) {
          const bool seen = (v[c >> 5] >> (c & 31)) & 1u;
          rr = seen ? -p.revisit_pen : sp * p.scale;
          v[c >> 5] |= 1u << (c & 31);
        }
        s[sCell] = __int_as_float(c);
        break;
      }
      case kRace: {
        const float d = field_sample(p, r[kOx], r[kOy], r[kOz]);
        float delta = s[sD] - d;
        const float clip = p.max_step * p.K;
        delta = fminf(fmaxf(delta, -clip), clip);
        rr = delta * p.scale - p.time_pen * p.K;
        if (p.speed_coef > 0) rr += p.speed_coef / 1000.0f * sp;
        if (p.speed_equiv > 0) rr += p.scale * p.speed_equiv * (sp - s[sSpeed]);
        if (ended) rr = 0.0f;
        if (goal) {
          rr += p.success_bonus;
          if (p.finish_k > 0) rr += p.finish_k * fmaxf(0.0f, p.finish_tref - (s[sTicks] + p.K) / 100.0f);
        }
        if (done && !goal) {
          rr -= p.fail_pen;
          if (p.speed_equiv > 0) rr -= p.scale * p.speed_equiv * s[sSpeed];   // death refund
        }
        s[sTicks] += p.K;
        const bool improved = d < s[sBest] - p.stall_eps;
        s[sBest] = fminf(s[sBest], d);
        s[sSince] = improved ? 0.0f : s[sSince] + p.K;
        s[sD] = d;
        break;
      }
    }
    if (p.mode == kAcro) {
      // style bonuses over the K ticks of this decision: ballistic flight =
      // velocity changed by gravity and small air-strafe increments only; a
      // ramp catch or floor is a large velocity change (reference
      // AcroCoverageReward, thresholds scaled from per tick to per decision)
      const float K = static_cast<float>(p.K);
      const float dvx = r[kVx] - s[sVx], dvy = r[kVy] - s[sVy], dvz = r[kVz] - s[sVz];
      const bool contact = fabsf(dvx) + fabsf(dvy) > 40.0f * K || fabsf(dvz + p.gravity_tick * K) > 12.0f * K;
      const bool grounded = r[kOnground] != 0.0f;
      const bool ballistic = !grounded && !contact;
      const float dyaw = fabsf(wrap180(r[kYaw] - s[sYaw]));
      const bool flight_end = s[sStreak] * K >= static_cast<float>(p.min_air) && (contact || grounded);
      const float spin_frac = fminf(s[sSpin], 360.0f * p.max_spins) / 360.0f;
      float style = flight_end ? p.spin_bonus * spin_frac : 0.0f;
      const float heading = atan2f(r[kVy], r[kVx]) * 57.29577951308232f;
      const bool backwards = fabsf(wrap180(r[kYaw] - heading)) >= 140.0f;
      if (flight_end && sp >= 300.0f && backwards) style += p.switch_bonus;
      if (!grounded && contact && sp >= 500.0f && backwards) style += p.back_bonus * K;
      s[sSpin] = ballistic ? s[sSpin] + (s[sStreak] > 0.0f ? fminf(dyaw, p.spin_rate_cap * K) : 0.0f) : 0.0f;
      s[sStreak] = ballistic ? s[sStreak] + 1.0f : 0.0f;
      if (!ended) rr += style;
      else { s[sSpin] = 0.0f; s[sStreak] = 0.0f; }
    }
    s[sYaw] = r[kYaw]; s[sVx] = r[kVx]; s[sVy] = r[kVy]; s[sVz] = r[kVz];
    if (p.mode != kRace && ended) rr = 0.0f;
    // curiosity: bonus from the counts as they stood before this decision
    if (p.int_coef > 0) {
      const int64_t key = curiosity_key(p, r);
      int64_t nk = -1;
      if (key != keys[i] && !ended) {
        ibonus = p.int_coef * rsqrtf(static_cast<float>(counts[bucket(p, key)]) + 1.0f);
        rr += ibonus;
        nk = key;
      }
      new_key[i] = nk;
      keys[i] = key;
    }
    if (boot) { rr += boot[i]; boot[i] = 0.0f; }        // truncation bootstrap gamma * V(s_T)
    rr += r[kBase];                                      // env-side (spline progress) reward
    rew_out[i] = rr;
    done_out[i] = ended ? 1.0f : 0.0f;
    s[sEpRet] += rr;
    s[sEpLen] += p.K;
    if (ended) {
      ep_done = 1.0f;
      ep_ret = s[sEpRet];
      ep_len = s[sEpLen];
      succ = goal ? 1.0f : 0.0f;
      fail = (done && !goal) ? 1.0f : 0.0f;
      trn = (!done) ? 1.0f : 0.0f;
      s[sEpRet] = 0.0f;
      s[sEpLen] = 0.0f;
      // re-anchor per-episode state on the new episode's spawn
      s[sBest] = sp;
      const float yaw = r[kYaw] * 0.017453292519943295f;
      s[sDirX] = cosf(yaw); s[sDirY] = sinf(yaw);
      s[sRefX] = r[kOx]; s[sRefY] = r[kOy];
      if (p.mode == kForward || p.mode == kBlend) s[sBest] = 0.0f;
      if (p.mode == kRace) { s[sBest] = s[sD]; s[sSince] = 0.0f; s[sTicks] = 0.0f; }
      if (p.mode == kCoverage || p.mode == kAcro) {
        uint32_t* v = visited + static_cast<int64_t>(i) * p.cov_words;
        for (int w = 0; w < p.cov_words; ++w) v[w] = 0;
        const int c = cov_cell(p, r);
        v[c >> 5] |= 1u << (c & 31);
        s[sCell] = __int_as_float(c);
      }
    }
    if (stall) {
      const bool kill = p.mode == kRace && p.stall_ticks > 0 && s[sSince] >= p.stall_ticks;
      if (kill) s[sSince] = 0.0f;
      stall[i] = kill ? 1 : 0;
    }
    s[sPx] = r[kOx]; s[sPy] = r[kOy]; s[sPz] = r[kOz];
    s[sSpeed] = sp;
  }
  // per-block reduction of episode statistics
  if (stats) {
    float vals[8] = {ep_done, ep_ret, ep_len, succ, fail, trn, ibonus, rr};
    for (int k = 0; k < 8; ++k)
      for (int o = 16; o; o >>= 1) vals[k] += __shfl_xor_sync(0xffffffffu, vals[k], o);
    if ((threadIdx.x & 31) == 0)
      for (int k = 0; k < 8; ++k) atomicAdd(stats + k, vals[k]);
  }
}

// phase 2: count increments (every entry counts once, duplicates included)
__global__ void count_kernel(RewardParams p, const int64_t* new_key, int* counts, int* delta) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= p.n) return;
  const int64_t k = new_key[i];
  if (k < 0) return;
  const uint32_t b = bucket(p, k);
  atomicAdd(counts + b, 1);
  if (delta) atomicAdd(delta + b, 1);
}

// proprioception features: out[i, j] = bf16(obs[i, idx[j]]) for j < nf, 0 beyond;
// with `extra`, column extra_col instead holds tanh(extra[i] / 0.1): the
// previous decision's reward fed back as an observation (reference
// --obs-reward, python/train_fast.py:2104-2113)
__global__ void features_kernel(const float* obs, int64_t ld_obs, const int* idx, int nf, int width, uint16_t* out,
                                int64_t ld_out, int n, const float* extra, int extra_col) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  for (int j = 0; j < width; ++j) {
    float v = 0.0f;
    if (j < nf) v = obs[i * ld_obs + idx[j]];
    if (extra && j == extra_col) v = tanhf(extra[i] * 10.0f);
    out[i * ld_out + j] = surfk::f32_to_bf16(v);
  }
}

// Keyed bijection of [0, n): a 4-round Feistel network on the smallest even
// bit width covering n, with cycle walking (Black & Rogaway, "Ciphers with
// arbitrary finite domains", CT-RSA 2002). Epoch permutations without a sort.
__device__ __forceinline__ uint32_t feistel_round(uint32_t x, uint32_t k) {
  x ^= k;
  x *= 0x9E3779B1u;
  x ^= x >> 15;
  x *= 0x85EBCA77u;
  x ^= x >> 13;
  return x;
}
__global__ void perm_kernel(int64_t* out, int64_t n, int half_bits, const uint64_t* key_ptr) {
  const uint64_t key = *key_ptr;
  const uint32_t mask = (1u << half_bits) - 1u;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    uint32_t x = static_cast<uint32_t>(i);
    do {
      uint32_t l = x >> half_bits, r = x & mask;
      for (int round = 0; round < 4; ++round) {
        const uint32_t f = feistel_round(r, static_cast<uint32_t>(key >> (16 * round)) * 0x2545F491u + round) & mask;
        const uint32_t nl = r;
        r = l ^ f;
        l = nl;
      }
      x = (l << half_bits) | r;
    } while (x >= static_cast<uint64_t>(n));
    out[i] = x;
  }
}

// The same keyed bijection over a pool whose size is read from device memory
// (it changes between iterations without a host round trip): out[i] =
// pool[pi(i)] for i < *count; the Feistel width follows *count.
__global__ void perm_pool_kernel(int64_t* out, const int64_t* pool, int64_t n_max, const int64_t* count,
                                 const uint64_t* key_ptr) {
  const int64_t n = *count < n_max ? *count : n_max;
  if (n <= 0) return;
  int bits = 2;
  while ((1ll << bits) < n) bits += 2;
  const int half_bits = bits / 2;
  const uint64_t key = *key_ptr;
  const uint32_t mask = (1u << half_bits) - 1u;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    uint32_t x = static_cast<uint32_t>(i);
    do {
      uint32_t l = x >> half_bits, r = x & mask;
      for (int round = 0; round < 4; ++round) {
        const uint32_t f = feistel_round(r, static_cast<uint32_t>(key >> (16 * round)) * 0x2545F491u + round) & mask;
        const uint32_t nl = r;
        r = l ^ f;
        l = nl;
      }
      x = (l << half_bits) | r;
    } while (x >= static_cast<uint64_t>(n));
    out[i] = pool[x];
  }
}

__global__ void bump_key_kernel(uint64_t* key) {
  uint64_t z = (*key += 0x9E3779B97F4A7C15ULL);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  *key = z ^ (z >> 27);
}

}  // namespace

SURF_EXPORT int surf_reward_params_size() { return static_cast<int>(sizeof(RewardParams)); }
SURF_EXPORT int surf_reward_state_floats() { return kStateFloats; }

// state: float [n*24] per env; keys: int64 [n] curiosity keys of the last
// decision. Every per-env pointer is indexed by the env's position in this
// call, so a contiguous group of envs is addressed by offsetting the pointers
// and setting p->n to the group size.
SURF_EXPORT int surf_reward_init(const RewardParams* p, const float* rec, int64_t ld, float* state, uint32_t* visited,
                                 int64_t* keys, void* stream) {
  reward_init_kernel<<<static_cast<int>(surfk::ceil_div(p->n, 128)), 128, 0, static_cast<cudaStream_t>(stream)>>>(
      *p, rec, ld, state, visited, keys);
  SURF_RETURN_LAUNCH();
}

// do_counts = 0 skips phase 2: a caller that splits the envs into groups
// runs phase 1 for every group, then surf_reward_counts once over all envs,
// so that every bonus of a decision reads the counts from before it.
SURF_EXPORT int surf_reward(const RewardParams* p, const float* rec, int64_t ld, float* state, uint32_t* visited,
                            int* counts, int* delta, float* boot, float* rew_out, float* done_out, uint8_t* stall,
                            int64_t* new_key, int64_t* keys, float* stats, int do_counts, void* stream) {
  auto s = static_cast<cudaStream_t>(stream);
  const int blocks = static_cast<int>(surfk::ceil_div(p->n, 128));
  reward_kernel<<<blocks, 128, 0, s>>>(*p, rec, ld, state, visited, counts, boot, rew_out, done_out, stall, new_key,
                                       keys, stats);
  if (p->int_coef > 0 && do_counts) count_kernel<<<blocks, 128, 0, s>>>(*p, new_key, counts, delta);
  SURF_RETURN_LAUNCH();
}

// phase 2 alone: count increments of the keys staged by phase 1 (p->n envs)
SURF_EXPORT int surf_reward_counts(const RewardParams* p, const int64_t* new_key, int* counts, int* delta,
                                   void* stream) {
  if (p->int_coef > 0)
    count_kernel<<<static_cast<int>(surfk::ceil_div(p->n, 128)), 128, 0, static_cast<cudaStream_t>(stream)>>>(
        *p, new_key, counts, delta);
  SURF_RETURN_LAUNCH();
}

SURF_EXPORT int surf_obs_features(const float* obs, int64_t ld_obs, const int* idx, int nf, int width, void* out,
                                  int64_t ld_out, int n, const float* extra, int extra_col, void* stream) {
  features_kernel<<<static_cast<int>(surfk::ceil_div(n, 128)), 128, 0, static_cast<cudaStream_t>(stream)>>>(
      obs, ld_obs, idx, nf, width, static_cast<uint16_t*>(out), ld_out, n, extra, extra_col);
  SURF_RETURN_LAUNCH();
}

// out[i] = pool[pi_key(i)] for i < *count (count <= n_max, read on the device);
// the key advances as in surf_permutation.
SURF_EXPORT int surf_permutation_pool(int64_t* out, const int64_t* pool, int64_t n_max, const int64_t* count,
                                      uint64_t* key, void* stream) {
  if (n_max < 1) return static_cast<int>(cudaErrorInvalidValue);
  auto s = static_cast<cudaStream_t>(stream);
  const int64_t blocks = surfk::ceil_div(n_max, 256);
  perm_pool_kernel<<<static_cast<int>(blocks < 148 * 16 ? blocks : 148 * 16), 256, 0, s>>>(out, pool, n_max, count, key);
  bump_key_kernel<<<1, 1, 0, s>>>(key);
  SURF_RETURN_LAUNCH();
}

// out[i] = pi_key(i), a permutation of [0, n); key read from device memory
// and then advanced (so a captured graph draws a fresh permutation per replay).
SURF_EXPORT int surf_permutation(int64_t* out, int64_t n, uint64_t* key, void* stream) {
  int bits = 2;
  while ((1ll << bits) < n) bits += 2;
  auto s = static_cast<cudaStream_t>(stream);
  perm_kernel<<<static_cast<int>(surfk::ceil_div(n, 256) < 148 * 16 ? surfk::ceil_div(n, 256) : 148 * 16), 256, 0, s>>>(
      out, n, bits / 2, key);
  bump_key_kernel<<<1, 1, 0, s>>>(key);
  SURF_RETURN_LAUNCH();
}
