// env_gpu.cu — the surf env batch on the GPU: one CUDA thread per env runs
// the same per-env rules as the host batch (EnvCore: pm_shared movement, hull
// traces, triggers, spline progress, autoreset; csrc/sim/env_core.hpp) over
// device copies of the map, so a rollout never leaves the device: actions are
// read from the sampler's output rows and the observation / record rows are
// written where the reward and camera kernels read them.
//
// The reference steps its envs on CPU threads (src/env.c:529-644) and ships
// observations to the GPU every decision; here the host only replays graphs.
// Parity: compiled with -fmad=false so every float expression rounds as in
// the host build (-ffp-contract=off); double sin/cos come from CUDA's libm,
// which agrees with the host's to within the last bit of a double and so, after
// the cast to float, almost always exactly (tests compare trajectories).
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "surf_cuda.cuh"
#include "../sim/env_core.hpp"

namespace {

using surf::EnvCore;
using surf::PlayerState;
using surf::RowOut;
using surf::Span;
using surf::StuckMemo;

constexpr int kMaxTreeDepth = surf::detail::kDescentDepthDevice;   // device descent stack (see collide.hpp)

struct GpuEnv {
  EnvCore core;                   // device pointers
  std::vector<void*> allocs;      // everything to free
  int n = 0;
  void* pool = nullptr;           // spawn pool (re-uploadable)
  int pool_cap = 0;
};

template <typename T>
int upload(Span<T>* dst, const Span<T>& src, GpuEnv* g) {
  dst->n = src.n;
  dst->p = nullptr;
  if (src.n <= 0) return 0;
  void* d = nullptr;
  cudaError_t e = cudaMalloc(&d, sizeof(T) * static_cast<size_t>(src.n));
  if (e != cudaSuccess) return static_cast<int>(e);
  g->allocs.push_back(d);
  e = cudaMemcpy(d, src.p, sizeof(T) * static_cast<size_t>(src.n), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return static_cast<int>(e);
  dst->p = static_cast<const T*>(d);
  return 0;
}

// A start-node grid of the world model (its cells array) to the device.
int upload_grid(surf::HullGrid* dst, const surf::HullGrid& src, GpuEnv* g) {
  *dst = src;
  dst->cells = nullptr;
  if (!src.cells) return 0;
  const size_t count = static_cast<size_t>(src.n[0]) * src.n[1] * src.n[2];
  void* d = nullptr;
  cudaError_t e = cudaMalloc(&d, sizeof(int32_t) * count);
  if (e != cudaSuccess) return static_cast<int>(e);
  g->allocs.push_back(d);
  e = cudaMemcpy(d, src.cells, sizeof(int32_t) * count, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return static_cast<int>(e);
  dst->cells = static_cast<const int32_t*>(d);
  return 0;
}

template <typename T>
int alloc_zero(T** dst, size_t count, GpuEnv* g) {
  void* d = nullptr;
  cudaError_t e = cudaMalloc(&d, sizeof(T) * (count ? count : 1));
  if (e != cudaSuccess) return static_cast<int>(e);
  g->allocs.push_back(d);
  e = cudaMemset(d, 0, sizeof(T) * (count ? count : 1));
  if (e != cudaSuccess) return static_cast<int>(e);
  *dst = static_cast<T*>(d);
  return 0;
}

// Deepest clip tree of any model and hull (the descent stack must hold it).
int max_tree_depth(const surf::MapView& m) {
  int best = 0;
  for (int mi = 0; mi < m.models.size(); ++mi)
    for (int h = 0; h < 4; ++h) {
      const surf::HullView v = m.hull(mi, h);
      const int d = surf::detail::hull_depth(v, v.first, kMaxTreeDepth);
      if (d > best) best = d;
    }
  return best;
}

__global__ void __launch_bounds__(128) step_k_kernel(EnvCore c, int lo, int hi, const int32_t* actions,
                                                     int64_t stride, int yaw_slot, int fail_slot, int k, RowOut obs,
                                                     RowOut term_obs, RowOut rec, RowOut term_rec) {
  const int i = lo + static_cast<int>(blockIdx.x * blockDim.x + threadIdx.x);
  if (i >= hi) return;
  c.step_k_one(i, actions + static_cast<int64_t>(i) * stride, yaw_slot, fail_slot, k, obs, term_obs, rec, term_rec,
               surf::envk::NoLidar());
}

// Spawn every env (reset_all) and write its first observation and record row.
__global__ void reset_kernel(EnvCore c, int n, uint64_t seed, RowOut obs, RowOut rec) {
  const int i = static_cast<int>(blockIdx.x * blockDim.x + threadIdx.x);
  if (i >= n) return;
  c.seed_and_reset(i, seed);
  const PlayerState& s = c.st[i];
  if (obs.ptr) c.write_obs(s, 0.0f, 0.0f, obs.row(i));
  if (rec.ptr) {
    float* o = rec.row(i);
    for (int k = 0; k < surf::kRecCols; ++k) o[k] = 0.0f;
    for (int k = 0; k < 3; ++k) { o[surf::kRecOrigin + k] = s.origin[k]; o[surf::kRecVel + k] = s.velocity[k]; }
    o[surf::kRecYaw] = s.yaw;
    o[surf::kRecPitch] = s.pitch;
    o[surf::kRecDucked] = static_cast<float>(s.ducked);    // (ground flag left 0, as the host trainer's reset)
  }
}

// Envs per block: the step is a chain of dependent loads per env (hull
// descents) whose lanes diverge (13 of 32 lanes active per instruction with
// full warps), so warps run few envs and every SM holds many of them: about
// 14 blocks per SM. Measured at 2048 envs: 2 or 4 envs per block 25M
// ticks/s, 8: 20M, 32: 12M; at 16,384 envs: 8 per block 121M, 32: 97M.
int threads_for(int n) {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        sms < 1)
      sms = 148;
  }
  static int forced = -1;                 // SURF_GENV_THREADS: a fixed block size (timing studies)
  if (forced < 0) {
    const char* e = std::getenv("SURF_GENV_THREADS");
    const int v = e ? std::atoi(e) : 0;
    forced = (v >= 1 && v <= 128) ? v : 0;
  }
  if (forced) return forced;
  int t = 2;
  while (t < 32 && t * sms * 14 < n) t *= 2;
  return t;
}

}  // namespace

SURF_EXPORT int surf_genv_core_size() { return static_cast<int>(sizeof(EnvCore)); }

// Build a GPU env from a host EnvCore (the bytes of the host batch's core, as
// returned by surfsim_core_bytes: host pointers valid in this process). The map
// arrays, progress spline and spawn pool are copied to the device; per-env
// state starts zeroed (call surf_genv_reset). *err receives a status code
// (0 ok, 1 lidar configured, 2 tree deeper than the device descent stack, or a
// cudaError_t + 100). Returns the handle or null.
SURF_EXPORT void* surf_genv_create(const void* host_core, int core_bytes, int* err) {
  *err = 0;
  if (core_bytes != static_cast<int>(sizeof(EnvCore))) { *err = 3; return nullptr; }
  EnvCore h;
  std::memcpy(&h, host_core, sizeof h);
  if (h.cfg.lidar_w > 0 && h.cfg.lidar_h > 0) { *err = 1; return nullptr; }
  if (max_tree_depth(h.map) > kMaxTreeDepth) { *err = 2; return nullptr; }
  auto* g = new GpuEnv();
  g->n = h.cfg.num_envs;
  EnvCore& c = g->core;
  c = h;
  for (auto& gr : c.map.world_grid) gr.cells = nullptr;   // host arrays until uploaded below
  c.ground = nullptr;                                      // the categorize cache is host-only
  int e = 0;
  e = e ? e : upload(&c.map.planes, h.map.planes, g);
  e = e ? e : upload(&c.map.clipnodes, h.map.clipnodes, g);
  e = e ? e : upload(&c.map.hull0, h.map.hull0, g);
  e = e ? e : upload(&c.map.models, h.map.models, g);
  e = e ? e : upload(&c.map.solids, h.map.solids, g);
  e = e ? e : upload(&c.map.volumes, h.map.volumes, g);
  e = e ? e : upload(&c.map.triggers, h.map.triggers, g);
  e = e ? e : upload(&c.map.spawns, h.map.spawns, g);
  for (int hh = 0; hh < 4; ++hh) e = e ? e : upload_grid(&c.map.world_grid[hh], h.map.world_grid[hh], g);
  e = e ? e : upload(&c.wp, h.wp, g);
  e = e ? e : upload(&c.cum, h.cum, g);
  e = e ? e : upload(&c.tang, h.tang, g);
  e = e ? e : upload(&c.tele_progress, h.tele_progress, g);
  e = e ? e : upload(&c.spawn_pool, h.spawn_pool, g);
  const size_t n = static_cast<size_t>(g->n);
  e = e ? e : alloc_zero(&c.st, n, g);
  e = e ? e : alloc_zero(&c.memo, n, g);
  e = e ? e : alloc_zero(&c.last_yd, n, g);
  e = e ? e : alloc_zero(&c.last_pd, n, g);
  e = e ? e : alloc_zero(&c.rng, n, g);
  e = e ? e : alloc_zero(&c.push_used, n * static_cast<size_t>(h.push_words > 0 ? h.push_words : 1), g);
  e = e ? e : alloc_zero(&c.goal_hit, n, g);
  e = e ? e : alloc_zero(&c.pending_fail, n, g);
  c.mover = surf::PlayerMove(c.map, h.cfg.phys);
  if (e) {
    for (void* p : g->allocs) cudaFree(p);
    delete g;
    *err = 100 + e;
    return nullptr;
  }
  return g;
}

SURF_EXPORT void surf_genv_destroy(void* handle) {
  auto* g = static_cast<GpuEnv*>(handle);
  if (!g) return;
  cudaDeviceSynchronize();
  for (void* p : g->allocs) cudaFree(p);
  delete g;
}

SURF_EXPORT int surf_genv_num_envs(void* handle) { return static_cast<GpuEnv*>(handle)->n; }

// Replace the spawn pool (host PlayerState rows), synchronously.
SURF_EXPORT int surf_genv_set_spawn_pool(void* handle, const void* pool, int count) {
  auto* g = static_cast<GpuEnv*>(handle);
  if (!pool || count < 1) { g->core.spawn_pool.p = nullptr; g->core.spawn_pool.n = 0; return 0; }
  if (count > g->pool_cap) {
    void* d = nullptr;
    cudaError_t e = cudaMalloc(&d, sizeof(PlayerState) * static_cast<size_t>(count));
    if (e != cudaSuccess) return static_cast<int>(e);
    g->allocs.push_back(d);
    g->pool = d;
    g->pool_cap = count;
  }
  cudaError_t e = cudaMemcpy(g->pool, pool, sizeof(PlayerState) * static_cast<size_t>(count), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return static_cast<int>(e);
  g->core.spawn_pool.p = static_cast<const PlayerState*>(g->pool);
  g->core.spawn_pool.n = count;
  return 0;
}

SURF_EXPORT int surf_genv_reset(void* handle, uint64_t seed, float* obs, int64_t obs_stride, float* rec,
                                int64_t rec_stride, void* stream) {
  auto* g = static_cast<GpuEnv*>(handle);
  RowOut o{obs, obs_stride}, r{rec, rec_stride};
  const int t = 64;
  reset_kernel<<<static_cast<unsigned>(surfk::ceil_div(g->n, t)), t, 0, static_cast<cudaStream_t>(stream)>>>(
      g->core, g->n, seed, o, r);
  SURF_RETURN_LAUNCH();
}

// K ticks of action repeat for envs [lo, hi): actions are int32 device rows of
// `stride` (slots 0..5 the discrete action; yaw_slot / fail_slot as in the host
// step_k); outputs are float32 device rows (any may be null).
SURF_EXPORT int surf_genv_step_k(void* handle, int lo, int hi, const int32_t* actions, int64_t stride, int yaw_slot,
                                 int fail_slot, int k, float* obs, int64_t obs_stride, float* term_obs,
                                 int64_t term_obs_stride, float* rec, int64_t rec_stride, float* term_rec,
                                 int64_t term_rec_stride, void* stream) {
  auto* g = static_cast<GpuEnv*>(handle);
  if (lo < 0) lo = 0;
  if (hi > g->n) hi = g->n;
  if (hi <= lo || !actions) return hi <= lo ? 0 : static_cast<int>(cudaErrorInvalidValue);
  if (k < 1) k = 1;
  const int t = threads_for(hi - lo);
  step_k_kernel<<<static_cast<unsigned>(surfk::ceil_div(hi - lo, t)), t, 0, static_cast<cudaStream_t>(stream)>>>(
      g->core, lo, hi, actions, stride, yaw_slot, fail_slot, k, RowOut{obs, obs_stride},
      RowOut{term_obs, term_obs_stride}, RowOut{rec, rec_stride}, RowOut{term_rec, term_rec_stride});
  SURF_RETURN_LAUNCH();
}

// Per-env player states, device <-> host (synchronous on `stream`).
SURF_EXPORT int surf_genv_get_states(void* handle, void* out, void* stream) {
  auto* g = static_cast<GpuEnv*>(handle);
  auto s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(out, g->core.st, sizeof(PlayerState) * static_cast<size_t>(g->n),
                                  cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  return static_cast<int>(e);
}

SURF_EXPORT int surf_genv_set_states(void* handle, const void* in, void* stream) {
  auto* g = static_cast<GpuEnv*>(handle);
  auto s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(g->core.st, in, sizeof(PlayerState) * static_cast<size_t>(g->n),
                                  cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  return static_cast<int>(e);
}

// Per-env RNG streams, device <-> host (checkpoints and parity tests).
SURF_EXPORT int surf_genv_rng(void* handle, uint64_t* host, int to_device, void* stream) {
  auto* g = static_cast<GpuEnv*>(handle);
  auto s = static_cast<cudaStream_t>(stream);
  const size_t bytes = sizeof(uint64_t) * static_cast<size_t>(g->n);
  cudaError_t e = to_device ? cudaMemcpyAsync(g->core.rng, host, bytes, cudaMemcpyHostToDevice, s)
                            : cudaMemcpyAsync(host, g->core.rng, bytes, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  return static_cast<int>(e);
}
