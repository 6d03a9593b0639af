// p2p.cu — data-parallel collectives over NVLink peer memory (sm_100a).
//
// One process per GPU. Every rank shares a few of its device buffers with
// the others through CUDA IPC (the gradient, the fp32 master parameters,
// their bf16 copy, the curiosity-count increments and a small sync block);
// the kernels below then read and write the peers' memory directly with
// plain loads/stores over NVLink/NVSwitch. No TMA, no multicast.
//
// Gradients cross NVLink in bf16: every rank publishes a bf16 copy of its
// fp32 gradient (the peers read it) and sums the W copies of its own shard
// in fp32, in rank order.
//
// Buckets (overlap with the backward pass): a contiguous range of the
// gradient that is final before the backward ends (the tower and FC weights,
// whose gradients come before the convolutions') is reduced by three small
// kernels launched on a side stream while the backward continues:
//   publish  convert the bucket of my gradient to bf16;
//   flag     release "bucket b published" to every peer;
//   reduce   wait for every peer's flag, then sum my shard's part of the
//            bucket from the W bf16 copies into my fp32 gradient, with
//            per-block sums of squares kept for the clip.
// None of them waits on another kernel of this GPU (only on peers' flags),
// and the reduce blocks wait independently, so they need no co-residency.
//
// Gradient step: ONE cooperative kernel (co-residency guaranteed by the
// cooperative launch attribute, so in-kernel grid barriers are safe; the
// launch is graph-capturable), for the rest of the gradient:
//   A  publish the bf16 copy of the ranges outside the buckets; the block
//      that finishes last tells every peer "my gradient is final"; every
//      block waits for all peers.
//   B  reduce-scatter of those ranges: rank r sums shard r of the W bf16
//      gradients (fixed rank order, fp32 accumulation, several 16-byte
//      groups per thread in flight) into its own fp32 gradient buffer;
//      per-block sums of squares (fp64); each block then arrives on a
//      counter and goes on (no grid-wide wait).
//   C  the block that arrives last adds the block sums in block order (and
//      the buckets' block sums after them) and publishes the shard's sum of
//      squares to every peer; every block
//      waits for all W shard norms and forms the clip coefficient (same
//      values, same order on every rank, so every rank clips identically).
//   D  Adam on the owned shard (m, v local); the new bf16 parameters are
//      pushed into every peer's buffers, the fp32 ones only for the tail
//      region the kernels read in fp32 (biases, log-std): the fp32 master
//      of the weight matrices stays sharded (16-byte stores). Each block
//      releases its stores at system scope and arrives on a second counter.
//   E  the last block to arrive raises "done" on every peer; every block
//      waits for all peers' "done" (every parameter pushed here, every peer
//      finished reading my gradient) and zeroes its part of the local
//      gradient.
// Moments: one block, all-gather of a few doubles + ordered local sum.
// Counts: one cooperative kernel: barrier-in, counts += every other rank's
//   increments, grid barrier, "done", wait, clear the local increments.
//
// Every wait (peer flags and grid barriers) polls with a bounded time
// (%globaltimer): a wait that runs out records an error code in the local
// sync block and the kernel returns, so a dead or stalled peer never hangs a
// GPU. Once an error is recorded every later collective kernel returns at
// once; the host reads the code after the step and raises.
//
// Semantics follow the data-parallel design of the reference
// (docs/ddp-plan.md:404-434 gradient sum after backward, before the clip;
// :133-147 global advantage moments; :174-225 count increments), realised
// here as fused peer-memory kernels instead of library all-reduces.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>

#include "surf_cuda.cuh"

namespace {

constexpr int kMaxW = 8;
constexpr int kMaxBlocks = 1024;
constexpr int kMaxMom = 256;
constexpr int kMaxB = 2;            // overlapped gradient buckets

// Sync block layout (uint64 words, one block per rank, zeroed at start).
enum : int {
  kSeqGrad = 0, kSeqMom = 1, kSeqCnt = 2, kErr = 3, kErrTarget = 4,
  kFlags = 16,                       // [6][kMaxW]
  kNormSlots = 64,                   // [2][kMaxW] doubles
  kBar = 96,                         // 8 grid barriers x (count, generation)
  kProf = 112,                       // phase timestamps of the last gradient step (block 0)
  kPartial = 128,                    // [kMaxBlocks] doubles
  kMomSlots = kPartial + kMaxBlocks, // [2][kMaxW][kMaxMom] doubles
  kBFlags = kMomSlots + 2 * kMaxW * kMaxMom,   // [kMaxB][kMaxW] "bucket published" flags
  kBPartial = kBFlags + kMaxB * kMaxW,         // [kMaxB][kMaxBlocks] doubles: bucket reduce block sums
  kSyncWords = kBPartial + kMaxB * kMaxBlocks,
};
enum : int { kFReady = 0, kFNorm = 1, kFDone = 2, kFMom = 3, kFCntReady = 4, kFCntDone = 5 };
enum : int { kBarGrad1 = 0, kBarGrad2 = 1, kBarCnt = 2, kBarGrad0 = 3 };

__host__ __device__ constexpr int flag_word(int f, int rank) { return kFlags + f * kMaxW + rank; }

struct Hyper { float lr, beta1, beta2, eps, max_norm, step; };

struct Plan {
  int rank = 0, world = 1;
  uint64_t timeout_ns = 0;
  uint64_t* sync = nullptr;                 // local sync block
  uint64_t* sync_peer[kMaxW] = {};          // every rank's sync block (peer[rank] = local)
  // gradient step
  int64_t n = 0, shard = 0;
  float* grad_peer[kMaxW] = {};
  uint16_t* g16_peer[kMaxW] = {};           // every rank's bf16 copy of its gradient (what peers read)
  int nb = 0;                               // overlapped buckets [b_lo, b_hi)
  int64_t b_lo[kMaxB] = {}, b_hi[kMaxB] = {};
  int nf = 1;                               // the rest: ranges [f_lo, f_hi), reduced by the step kernel
  int64_t f_lo[kMaxB + 1] = {}, f_hi[kMaxB + 1] = {};
  int bgrid = 296;                          // blocks of a bucket reduce
  float* p_peer[kMaxW] = {};
  uint16_t* p16_peer[kMaxW] = {};
  float* m = nullptr;
  float* v = nullptr;
  float* hyper = nullptr;
  int64_t push32_from = 0;                  // fp32 parameters pushed to peers only from this index on
  int coop_grid = 148;                      // co-resident blocks of the cooperative kernels
  // timing studies only (SURF_P2P_DBG, read at plan creation): bit 0 skips
  // the reduce-scatter loop, bit 1 the Adam loop, bit 2 gives the second grid
  // barrier a device-scope fence instead of a system-scope one (results are
  // then unordered across GPUs), bit 3 skips the gradient clear
  int dbg = 0;
  // counts merge
  int64_t cn = 0;
  int* counts = nullptr;
  int* delta_peer[kMaxW] = {};
};

// ---- memory-model helpers (inline PTX) -----------------------------------------------------
__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_sys(double* p, double v) {
  asm volatile("st.relaxed.sys.global.f64 [%0], %1;" ::"l"(p), "d"(v) : "memory");
}
__device__ __forceinline__ double ld_relaxed_sys(const double* p) {
  double v;
  asm volatile("ld.relaxed.sys.global.f64 %0, [%1];" : "=d"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Record the first error (code, and the sequence number it happened at).
__device__ void set_error(uint64_t* sync, uint64_t code, uint64_t target) {
  if (atomicCAS(reinterpret_cast<unsigned long long*>(sync + kErr), 0ull, static_cast<unsigned long long>(code)) == 0ull)
    sync[kErrTarget] = target;
}

// Poll until *flag >= target; false (error recorded) after timeout_ns or when
// another block of this rank already recorded an error.
__device__ bool wait_flag(const uint64_t* flag, uint64_t target, uint64_t* sync, uint64_t timeout_ns, uint64_t code) {
  if (ld_acquire_sys(flag) >= target) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    __nanosleep(128);
    if (ld_acquire_sys(flag) >= target) return true;
    if ((it & 31u) == 0u) {
      if (ld_relaxed_sys_u64(sync + kErr) != 0ull) return false;
      if (globaltimer() - t0 > timeout_ns || it > 0x7fffffffu) {
        set_error(sync, code, target);
        return false;
      }
    }
  }
}

// Every thread t < world waits for flag f of rank t; the block agrees on the
// result. Returns false if any wait failed (or an error is already recorded).
__device__ bool block_wait_all(const Plan& P, int f, uint64_t target, uint64_t code) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = ld_relaxed_sys_u64(P.sync + kErr) == 0ull;
  __syncthreads();
  if (ok && static_cast<int>(threadIdx.x) < P.world) {
    if (!wait_flag(P.sync + flag_word(f, threadIdx.x), target, P.sync, P.timeout_ns, code + threadIdx.x)) ok = 0;
  }
  __syncthreads();
  return ok != 0;
}

// Every thread t < world waits for word base + t of the local sync block.
__device__ bool block_wait_words(const Plan& P, int base, uint64_t target, uint64_t code) {
  __shared__ int okw;
  if (threadIdx.x == 0) okw = ld_relaxed_sys_u64(P.sync + kErr) == 0ull;
  __syncthreads();
  if (okw && static_cast<int>(threadIdx.x) < P.world) {
    if (!wait_flag(P.sync + base + threadIdx.x, target, P.sync, P.timeout_ns, code + threadIdx.x)) okw = 0;
  }
  __syncthreads();
  return okw != 0;
}

__device__ __forceinline__ double block_sum(double s) {
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  __shared__ double red[32];
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = s;
  __syncthreads();
  double t = 0.0;
  if (threadIdx.x == 0)
    for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) t += red[i];
  __syncthreads();
  return t;   // valid in thread 0
}

__device__ __forceinline__ uint64_t ld_acquire_gpu(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Grid-wide barrier of a cooperative launch (sense by generation counter),
// bounded like every other wait. `fence_sys` makes this block's earlier
// stores (peer stores included) visible system-wide before it arrives.
__device__ bool grid_barrier(uint64_t* sync, int slot, bool fence_sys, uint64_t timeout_ns, uint64_t code,
                             uint64_t target) {
  __shared__ int ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    ok = 1;
    unsigned long long* cnt = reinterpret_cast<unsigned long long*>(sync + kBar + 2 * slot);
    unsigned long long* gen = cnt + 1;
    const uint64_t g = ld_acquire_gpu(reinterpret_cast<uint64_t*>(gen));
    // release of this block's writes (system scope when peers will read them)
    if (fence_sys) fence_acq_rel_sys();
    else fence_acq_rel_gpu();
    if (atomicAdd(cnt, 1ull) == gridDim.x - 1) {
      atomicExch(cnt, 0ull);
      fence_acq_rel_gpu();
      atomicAdd(gen, 1ull);
    } else {
      const uint64_t t0 = globaltimer();
      for (uint32_t it = 1; ld_acquire_gpu(reinterpret_cast<uint64_t*>(gen)) == g; ++it) {
        if ((it & 63u) == 0u) {
          if (ld_relaxed_sys_u64(sync + kErr) != 0ull) { ok = 0; break; }
          if (globaltimer() - t0 > timeout_ns) { set_error(sync, code, target); ok = 0; break; }
        }
      }
    }
  }
  __syncthreads();
  return ok != 0;
}

// One-shot arrival counter of a cooperative launch: every block arrives once
// and goes on without waiting; the block that arrives last (the result is
// block-uniform) has acquired every other block's writes made before their
// arrival, and resets the counter for the kernel's next launch. `fence_sys`
// releases this block's writes at system scope (peer stores made here).
__device__ bool arrive_last(uint64_t* sync, int slot, bool fence_sys) {
  __shared__ int last;
  __syncthreads();
  if (threadIdx.x == 0) {
    if (fence_sys) fence_acq_rel_sys();
    else fence_acq_rel_gpu();
    unsigned long long* cnt = reinterpret_cast<unsigned long long*>(sync + kBar + 2 * slot);
    last = atomicAdd(cnt, 1ull) == gridDim.x - 1 ? 1 : 0;
    if (last) {
      fence_acq_rel_gpu();
      atomicExch(cnt, 0ull);
    }
  }
  __syncthreads();
  return last != 0;
}

__device__ __forceinline__ void prof_mark(const Plan& P, int k) {
  if (blockIdx.x == 0 && threadIdx.x == 0) P.sync[kProf + k] = globaltimer();
}

// bf16 copy of gradient[lo, hi) (lo, hi multiples of 8) into this rank's published buffer
__device__ void publish_range(const Plan& P, int64_t lo, int64_t hi, int64_t tid, int64_t stride) {
  const float* g = P.grad_peer[P.rank];
  uint16_t* o = P.g16_peer[P.rank];
  for (int64_t j = lo / 8 + tid; j < hi / 8; j += stride) {
    const float4 a = reinterpret_cast<const float4*>(g)[2 * j];
    const float4 b = reinterpret_cast<const float4*>(g)[2 * j + 1];
    reinterpret_cast<uint4*>(o)[j] = make_uint4(surfk::pack_bf16x2(a.x, a.y), surfk::pack_bf16x2(a.z, a.w),
                                                surfk::pack_bf16x2(b.x, b.y), surfk::pack_bf16x2(b.z, b.w));
  }
}

__device__ __forceinline__ void add_bf16x8(float* acc, const uint4& w) {
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    acc[2 * k] += __uint_as_float(u[k] << 16);
    acc[2 * k + 1] += __uint_as_float(u[k] & 0xFFFF0000u);
  }
}

// fp32 sum of the W gradients over [lo, hi) (multiples of 8), rank order
// 0..W-1, into this rank's fp32 gradient: the peers' terms from their
// published bf16 copies, this rank's own term in fp32 (each element is
// reduced by its owner only, so the mix is the same wherever it is read);
// returns the thread's sum of squares. kU 16-byte groups per peer in
// flight per thread.
template <int W, int kU>
__device__ double reduce_range(const Plan& P, int64_t lo, int64_t hi, int64_t tid, int64_t stride) {
  double ss = 0.0;
  float* mine = P.grad_peer[P.rank];
  const int64_t j_lo = lo / 8, j_hi = hi / 8;
  for (int64_t j0 = j_lo + tid; j0 < j_hi; j0 += stride * kU) {
    uint4 v[W][kU];
    float4 own[2][kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t j = j0 + u * stride;
      if (j < j_hi) {
#pragma unroll
        for (int q = 0; q < W; ++q)
          if (q != P.rank) v[q][u] = reinterpret_cast<const uint4*>(P.g16_peer[q])[j];
        own[0][u] = reinterpret_cast<const float4*>(mine)[2 * j];
        own[1][u] = reinterpret_cast<const float4*>(mine)[2 * j + 1];
      }
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t j = j0 + u * stride;
      if (j < j_hi) {
        float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int q = 0; q < W; ++q) {
          if (q == P.rank) {
            a[0] += own[0][u].x; a[1] += own[0][u].y; a[2] += own[0][u].z; a[3] += own[0][u].w;
            a[4] += own[1][u].x; a[5] += own[1][u].y; a[6] += own[1][u].z; a[7] += own[1][u].w;
          } else {
            add_bf16x8(a, v[q][u]);
          }
        }
        reinterpret_cast<float4*>(mine)[2 * j] = make_float4(a[0], a[1], a[2], a[3]);
        reinterpret_cast<float4*>(mine)[2 * j + 1] = make_float4(a[4], a[5], a[6], a[7]);
#pragma unroll
        for (int k = 0; k < 8; ++k) ss += static_cast<double>(a[k]) * a[k];
      }
    }
  }
  return ss;
}

// ---- overlapped buckets ----------------------------------------------------------------------
__global__ void __launch_bounds__(128) bucket_publish_kernel(Plan P, int b) {
  if (ld_relaxed_sys_u64(P.sync + kErr) != 0ull) return;
  publish_range(P, P.b_lo[b], P.b_hi[b], blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x,
                static_cast<int64_t>(gridDim.x) * blockDim.x);
}

// runs after the publish kernel in stream order: its bf16 copy is complete
__global__ void bucket_flag_kernel(Plan P, int b) {
  if (ld_relaxed_sys_u64(P.sync + kErr) != 0ull) return;
  const uint64_t target = P.sync[kSeqGrad] + 1;
  fence_acq_rel_sys();
  if (static_cast<int>(threadIdx.x) < P.world)
    st_release_sys(P.sync_peer[threadIdx.x] + kBFlags + b * kMaxW + P.rank, target);
}

// small blocks and grid (kBucketThreads x Plan::bgrid): the bucket kernels
// run beside the backward's kernels (one 320-thread CTA per SM) instead of
// displacing them
constexpr int kBucketThreads = 128;

template <int W>
__global__ void __launch_bounds__(kBucketThreads) bucket_reduce_kernel(Plan P, int b) {
  constexpr int kU = W <= 2 ? 2 : 1;             // registers: <= 88 per thread at every W
  double* part = reinterpret_cast<double*>(P.sync + kBPartial) + b * kMaxBlocks;
  if (ld_relaxed_sys_u64(P.sync + kErr) != 0ull) return;
  const uint64_t target = P.sync[kSeqGrad] + 1;
  if (!block_wait_words(P, kBFlags + b * kMaxW, target, 0x800 + 0x10 * b)) return;
  const int64_t s_lo = static_cast<int64_t>(P.rank) * P.shard;
  const int64_t s_hi = s_lo + P.shard < P.n ? s_lo + P.shard : P.n;
  const int64_t lo = s_lo > P.b_lo[b] ? s_lo : P.b_lo[b];
  const int64_t hi = s_hi < P.b_hi[b] ? s_hi : P.b_hi[b];
  double ss = 0.0;
  if (hi > lo && !(P.dbg & 1))
    ss = reduce_range<W, kU>(P, lo, hi, blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x,
                             static_cast<int64_t>(gridDim.x) * blockDim.x);
  const double bs = block_sum(ss);
  if (threadIdx.x == 0) part[blockIdx.x] = bs;
}

// ---- gradient step ---------------------------------------------------------------------------
// W = world size (compile-time, so the peer loops hold exactly W float4 per
// group in registers). Every thread keeps kU float4 groups per peer in flight
// at once: the reduce-scatter is a read of (W-1)/W of the gradient over
// NVLink, and its rate is bytes in flight / round-trip latency.
template <int W>
__global__ void __launch_bounds__(256) grad_step_kernel(Plan P) {
  constexpr int kU = W <= 1 ? 8 : (W == 2 ? 4 : (W <= 4 ? 2 : 1));   // groups per thread per round (reduce-scatter)
  constexpr int kUA = 4;                                              // groups per thread per round (Adam)
  uint64_t* sync = P.sync;
  if (ld_relaxed_sys_u64(sync + kErr) != 0ull) return;
  const uint64_t target = sync[kSeqGrad] + 1;
  const int par = static_cast<int>(target & 1);
  const int64_t tid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  prof_mark(P, 0);
  // A: publish the bf16 copy of the ranges outside the buckets; the last
  // block to finish releases "ready" to every peer (system-scope release of
  // every block's copy), then every block waits for all peers
  for (int f = 0; f < P.nf; ++f) publish_range(P, P.f_lo[f], P.f_hi[f], tid, stride);
  if (arrive_last(sync, kBarGrad0, true) && static_cast<int>(threadIdx.x) < P.world)
    st_release_sys(P.sync_peer[threadIdx.x] + flag_word(kFReady, P.rank), target);
  if (!block_wait_all(P, kFReady, target, 0x100)) return;
  prof_mark(P, 1);

  const int64_t lo = static_cast<int64_t>(P.rank) * P.shard;
  const int64_t hi = lo + P.shard < P.n ? lo + P.shard : P.n;
  const int64_t cnt = hi > lo ? hi - lo : 0;
  // 4-element groups (the shard start is 32-byte aligned) for Adam below
  const int64_t n4 = cnt >> 2;
  float* mine = P.grad_peer[P.rank];
  // B: reduce-scatter of the owned shard outside the buckets (rank order
  // 0..W-1 in every sum, fp32 accumulation of the bf16 copies)
  double ss = 0.0;
  for (int f = 0; f < P.nf && !(P.dbg & 1); ++f) {
    const int64_t a = lo > P.f_lo[f] ? lo : P.f_lo[f];
    const int64_t e = hi < P.f_hi[f] ? hi : P.f_hi[f];
    if (e > a) ss += reduce_range<W, kU>(P, a, e, tid, stride);
  }
  const double bs = block_sum(ss);
  double* partial = reinterpret_cast<double*>(sync + kPartial);
  if (threadIdx.x == 0) partial[blockIdx.x] = bs;
  const bool last1 = arrive_last(sync, kBarGrad1, false);
  prof_mark(P, 2);
  // C: shard norm out (by the block that finished the reduce-scatter last),
  // all norms in
  if (last1) {
    // ordered (deterministic) sum of the block partials by the whole block:
    // thread t adds blocks t, t+256, ... then a fixed-shape tree
    double part = 0.0;
    for (unsigned b = threadIdx.x; b < gridDim.x; b += blockDim.x) part += partial[b];
    // the overlapped buckets' block sums, bucket by bucket (their kernels
    // finished before this one: stream order)
    for (int bk = 0; bk < P.nb; ++bk) {
      const double* bp = reinterpret_cast<const double*>(sync + kBPartial) + bk * kMaxBlocks;
      for (int b = threadIdx.x; b < P.bgrid; b += blockDim.x) part += bp[b];
    }
    const double tot_b = block_sum(part);
    __shared__ double s_tot;
    if (threadIdx.x == 0) s_tot = tot_b;
    __syncthreads();
    // one thread per peer: its norm slot, then its flag with release order
    // (a single thread releasing to every peer in turn would serialise one
    // system-scope fence per peer and skew the peers' wake-ups)
    if (static_cast<int>(threadIdx.x) < P.world) {
      const int q = threadIdx.x;
      st_relaxed_sys(reinterpret_cast<double*>(P.sync_peer[q] + kNormSlots) + par * kMaxW + P.rank, s_tot);
      st_release_sys(P.sync_peer[q] + flag_word(kFNorm, P.rank), target);
    }
  }
  if (!block_wait_all(P, kFNorm, target, 0x200)) return;
  prof_mark(P, 3);
  __shared__ float s_coef;
  const Hyper* h = reinterpret_cast<const Hyper*>(P.hyper);
  if (threadIdx.x == 0) {
    const double* slots = reinterpret_cast<const double*>(sync + kNormSlots) + par * kMaxW;
    double tot = 0.0;
    for (int q = 0; q < P.world; ++q) tot += ld_relaxed_sys(slots + q);
    const float norm = static_cast<float>(sqrt(tot));
    s_coef = h->max_norm > 0.0f ? fminf(1.0f, h->max_norm / (norm + 1e-6f)) : 1.0f;
  }
  __syncthreads();
  // D: Adam on the owned shard, push the new parameters everywhere
  const float coef = s_coef, b1 = h->beta1, b2 = h->beta2, t = h->step + 1.0f, eps = h->eps;
  const float bc1 = 1.0f - powf(b1, t), bc2 = 1.0f - powf(b2, t);
  const float lr_t = h->lr / bc1, rbc2 = rsqrtf(bc2);
  const float* pl = P.p_peer[P.rank];
  auto adam1 = [&](float gi, float& mi, float& vi, float pi) {
    gi *= coef;
    mi = b1 * mi + (1.0f - b1) * gi;
    vi = b2 * vi + (1.0f - b2) * gi * gi;
    return pi - lr_t * mi / (sqrtf(vi) * rbc2 + eps);
  };
  auto adam4 = [&](const float4 g4, float4& m4, float4& v4, float4 p4) {
    p4.x = adam1(g4.x, m4.x, v4.x, p4.x);
    p4.y = adam1(g4.y, m4.y, v4.y, p4.y);
    p4.z = adam1(g4.z, m4.z, v4.z, p4.z);
    p4.w = adam1(g4.w, m4.w, v4.w, p4.w);
    return p4;
  };
  auto pack2 = [](float a, float b) { return surfk::pack_bf16x2(a, b); };
  for (int64_t j0 = tid; j0 < ((P.dbg & 2) ? 0 : n4); j0 += stride * kUA) {
    float4 g4[kUA], m4[kUA], v4[kUA], p4[kUA];
#pragma unroll
    for (int u = 0; u < kUA; ++u) {
      const int64_t j = j0 + u * stride;
      if (j < n4) {
        const int64_t i = lo + 4 * j;
        g4[u] = *reinterpret_cast<const float4*>(mine + i);
        m4[u] = *reinterpret_cast<const float4*>(P.m + i);
        v4[u] = *reinterpret_cast<const float4*>(P.v + i);
        p4[u] = *reinterpret_cast<const float4*>(pl + i);
      }
    }
#pragma unroll
    for (int u = 0; u < kUA; ++u) {
      const int64_t j = j0 + u * stride;
      if (j < n4) {
        const int64_t i = lo + 4 * j;
        const float4 p0 = adam4(g4[u], m4[u], v4[u], p4[u]);
        *reinterpret_cast<float4*>(P.m + i) = m4[u];
        *reinterpret_cast<float4*>(P.v + i) = v4[u];
        const uint2 b = make_uint2(pack2(p0.x, p0.y), pack2(p0.z, p0.w));
        const bool all32 = i >= P.push32_from;      // 64-aligned region boundary: never inside a group of 4
#pragma unroll
        for (int q = 0; q < W; ++q) {
          if (all32 || q == P.rank) *reinterpret_cast<float4*>(P.p_peer[q] + i) = p0;
          *reinterpret_cast<uint2*>(P.p16_peer[q] + i) = b;
        }
      }
    }
  }
  for (int64_t i = lo + 4 * n4 + tid; i < hi; i += stride) {
    float mi = P.m[i], vi = P.v[i];
    const float pi = adam1(mine[i], mi, vi, pl[i]);
    P.m[i] = mi;
    P.v[i] = vi;
    const uint16_t b = surfk::f32_to_bf16(pi);
    for (int q = 0; q < W; ++q) {
      if (i >= P.push32_from || q == P.rank) P.p_peer[q][i] = pi;
      P.p16_peer[q][i] = b;
    }
  }
  const bool last2 = arrive_last(sync, kBarGrad2, !(P.dbg & 4));
  prof_mark(P, 4);
  // E: done out (by the block that pushed last), all done in, clear the
  // local gradient (every peer finished reading it before it published its
  // norm; "done" also says its parameters have landed here)
  if (last2) {
    if (static_cast<int>(threadIdx.x) < P.world)
      st_release_sys(P.sync_peer[threadIdx.x] + flag_word(kFDone, P.rank), target);
    if (threadIdx.x == 0) {
      reinterpret_cast<Hyper*>(P.hyper)->step = t;  // every block read the old step before it arrived
      sync[kSeqGrad] = target;
    }
  }
  if (!block_wait_all(P, kFDone, target, 0x300)) return;
  prof_mark(P, 5);
  const int64_t nv = (P.dbg & 8) ? 0 : P.n >> 2;
  for (int64_t j = tid; j < nv; j += stride) reinterpret_cast<float4*>(mine)[j] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int64_t i = 4 * nv + tid; i < P.n; i += stride) mine[i] = 0.0f;
}

// ---- moments (tiny all-reduce, one block) ---------------------------------------------------
__global__ void __launch_bounds__(256) moments_kernel(Plan P, double* mom, int cnt) {
  uint64_t* sync = P.sync;
  if (ld_relaxed_sys_u64(sync + kErr) != 0ull) return;
  const uint64_t target = sync[kSeqMom] + 1;
  const int par = static_cast<int>(target & 1);
  for (int i = threadIdx.x; i < P.world * cnt; i += blockDim.x) {
    const int q = i / cnt, k = i % cnt;
    double* dst = reinterpret_cast<double*>(P.sync_peer[q] + kMomSlots) + (par * kMaxW + P.rank) * kMaxMom + k;
    st_relaxed_sys(dst, mom[k]);
  }
  __threadfence_system();
  __syncthreads();
  if (static_cast<int>(threadIdx.x) < P.world)
    st_release_sys(P.sync_peer[threadIdx.x] + flag_word(kFMom, P.rank), target);
  if (!block_wait_all(P, kFMom, target, 0x400)) return;
  const double* slots = reinterpret_cast<const double*>(sync + kMomSlots) + par * kMaxW * kMaxMom;
  for (int k = threadIdx.x; k < cnt; k += blockDim.x) {
    double s = 0.0;
    for (int q = 0; q < P.world; ++q) s += ld_relaxed_sys(slots + q * kMaxMom + k);
    mom[k] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) sync[kSeqMom] = target;
}

// ---- curiosity count merge -----------------------------------------------------------------
__global__ void __launch_bounds__(256) counts_merge_kernel(Plan P) {
  uint64_t* sync = P.sync;
  if (ld_relaxed_sys_u64(sync + kErr) != 0ull) return;
  const uint64_t target = sync[kSeqCnt] + 1;
  if (blockIdx.x == 0 && static_cast<int>(threadIdx.x) < P.world)
    st_release_sys(P.sync_peer[threadIdx.x] + flag_word(kFCntReady, P.rank), target);
  if (!block_wait_all(P, kFCntReady, target, 0x500)) return;
  const int64_t nv = P.cn >> 2;
  const int64_t tid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t j = tid; j < nv; j += stride) {
    int4 acc = reinterpret_cast<const int4*>(P.counts)[j];
#pragma unroll
    for (int q = 0; q < kMaxW; ++q) {
      if (q < P.world && q != P.rank) {
        const int4 d = reinterpret_cast<const int4*>(P.delta_peer[q])[j];
        acc.x += d.x; acc.y += d.y; acc.z += d.z; acc.w += d.w;
      }
    }
    reinterpret_cast<int4*>(P.counts)[j] = acc;
  }
  for (int64_t i = 4 * nv + tid; i < P.cn; i += stride) {
    int acc = P.counts[i];
    for (int q = 0; q < P.world; ++q)
      if (q != P.rank) acc += P.delta_peer[q][i];
    P.counts[i] = acc;
  }
  if (!grid_barrier(sync, kBarCnt, true, P.timeout_ns, 0x730, target)) return;
  if (blockIdx.x == 0 && static_cast<int>(threadIdx.x) < P.world)
    st_release_sys(P.sync_peer[threadIdx.x] + flag_word(kFCntDone, P.rank), target);
  if (blockIdx.x == 0 && threadIdx.x == 0) sync[kSeqCnt] = target;
  if (!block_wait_all(P, kFCntDone, target, 0x600)) return;
  int* d = P.delta_peer[P.rank];
  for (int64_t j = tid; j < nv; j += stride) reinterpret_cast<int4*>(d)[j] = make_int4(0, 0, 0, 0);
  for (int64_t i = 4 * nv + tid; i < P.cn; i += stride) d[i] = 0;
}

using BucketKernel = void (*)(Plan, int);
BucketKernel bucket_kernel_for(int world) {
  switch (world) {
    case 1: return bucket_reduce_kernel<1>;
    case 2: return bucket_reduce_kernel<2>;
    case 3: return bucket_reduce_kernel<3>;
    case 4: return bucket_reduce_kernel<4>;
    case 5: return bucket_reduce_kernel<5>;
    case 6: return bucket_reduce_kernel<6>;
    case 7: return bucket_reduce_kernel<7>;
    default: return bucket_reduce_kernel<8>;
  }
}

using GradKernel = void (*)(Plan);
GradKernel grad_kernel_for(int world) {
  switch (world) {
    case 1: return grad_step_kernel<1>;
    case 2: return grad_step_kernel<2>;
    case 3: return grad_step_kernel<3>;
    case 4: return grad_step_kernel<4>;
    case 5: return grad_step_kernel<5>;
    case 6: return grad_step_kernel<6>;
    case 7: return grad_step_kernel<7>;
    default: return grad_step_kernel<8>;
  }
}

// Cooperative launch (all blocks co-resident, so grid barriers are safe).
template <typename K>
int launch_coop(K kernel, int grid, cudaStream_t s, const Plan& P) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return static_cast<int>(cudaLaunchKernelEx(&cfg, kernel, P));
}


// ---- IPC bookkeeping -----------------------------------------------------------------------
std::mutex g_mu;
std::map<std::string, void*> g_opened;    // handle bytes -> mapped base (one mapping per allocation)

}  // namespace

SURF_EXPORT int surf_p2p_sync_words() { return kSyncWords; }
SURF_EXPORT int surf_p2p_max_world() { return kMaxW; }
SURF_EXPORT int surf_p2p_max_moments() { return kMaxMom; }

// Handle of the allocation containing p (64 bytes) and p's offset in it.
SURF_EXPORT int surf_ipc_handle(const void* p, void* handle_out, int64_t* offset_out) {
  CUdeviceptr base = 0;
  size_t size = 0;
  CUresult r = cuMemGetAddressRange(&base, &size, reinterpret_cast<CUdeviceptr>(p));
  if (r != CUDA_SUCCESS) return 1000 + static_cast<int>(r);
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return static_cast<int>(e);
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<int64_t>(reinterpret_cast<uintptr_t>(p) - static_cast<uintptr_t>(base));
  return 0;
}

// Map a peer's allocation (once per allocation) and return base + offset.
SURF_EXPORT int surf_ipc_open(const void* handle, int64_t offset, void** ptr_out) {
  std::lock_guard<std::mutex> lk(g_mu);
  const std::string key(static_cast<const char*>(handle), sizeof(cudaIpcMemHandle_t));
  auto it = g_opened.find(key);
  void* base = nullptr;
  if (it != g_opened.end()) {
    base = it->second;
  } else {
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return static_cast<int>(e);
    g_opened[key] = base;
  }
  *ptr_out = static_cast<char*>(base) + offset;
  return 0;
}

// Unmap every peer allocation opened by this process.
SURF_EXPORT int surf_ipc_close_all() {
  std::lock_guard<std::mutex> lk(g_mu);
  int rc = 0;
  for (auto& kv : g_opened) {
    cudaError_t e = cudaIpcCloseMemHandle(kv.second);
    if (e != cudaSuccess && rc == 0) rc = static_cast<int>(e);
  }
  g_opened.clear();
  return rc;
}

// Host-side plan (no device memory is allocated here).
SURF_EXPORT void* surf_p2p_create(int rank, int world, void* const* sync_peers, double timeout_s) {
  if (world < 1 || world > kMaxW || rank < 0 || rank >= world) return nullptr;
  Plan* p = new Plan();
  p->rank = rank;
  p->world = world;
  p->timeout_ns = static_cast<uint64_t>(timeout_s * 1e9);
  for (int q = 0; q < world; ++q) p->sync_peer[q] = static_cast<uint64_t*>(sync_peers[q]);
  p->sync = p->sync_peer[rank];
  int dev = 0, sms = 148, per_sm = 1, per_sm2 = 1;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // the largest instantiation bounds the co-resident blocks of all of them
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, grad_step_kernel<kMaxW>, 256, 0);
  for (int w = 1; w < kMaxW; ++w) {
    int b = 1;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, grad_kernel_for(w), 256, 0);
    if (b < per_sm) per_sm = b;
  }
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm2, counts_merge_kernel, 256, 0);
  const int m = per_sm < per_sm2 ? per_sm : per_sm2;
  p->coop_grid = sms * (m < 2 ? (m < 1 ? 1 : m) : 2);
  // SURF_P2P_BLOCKS_PER_SM (1 or 2) overrides the blocks per SM (tuning studies)
  if (const char* e = std::getenv("SURF_P2P_BLOCKS_PER_SM")) {
    const int b = std::atoi(e);
    if (b >= 1 && b <= m) p->coop_grid = sms * b;
  }
  if (p->coop_grid > kMaxBlocks) p->coop_grid = kMaxBlocks;
  p->bgrid = sms / 2 > 0 ? sms / 2 : 1;        // bucket kernels: a small footprint beside the backward
  if (const char* e = std::getenv("SURF_P2P_BUCKET_BLOCKS")) {
    const int b = std::atoi(e);
    if (b >= 1 && b <= kMaxBlocks) p->bgrid = b;
  }
  if (const char* e = std::getenv("SURF_P2P_DBG")) p->dbg = std::atoi(e);
  return p;
}

SURF_EXPORT void surf_p2p_destroy(void* plan) { delete static_cast<Plan*>(plan); }

// Shard = ceil(n / world) rounded up to 8 elements; every buffer must be
// 16-byte aligned (torch allocations are).
// push32_from: parameters below this index keep their fp32 master on the
// owning rank only (peers receive the bf16 copy); from it on, every rank
// receives fp32 too. Must be a multiple of 8 (0 = replicate everything).
SURF_EXPORT int surf_p2p_set_grad(void* plan, int64_t n, void* const* grad_peers, void* const* p_peers,
                                  void* const* p16_peers, float* m, float* v, float* hyper, int64_t push32_from) {
  Plan* P = static_cast<Plan*>(plan);
  if (push32_from < 0 || push32_from % 8) return static_cast<int>(cudaErrorInvalidValue);
  if (n % 8) return static_cast<int>(cudaErrorInvalidValue);   // 16-byte bf16 groups
  P->n = n;
  P->push32_from = push32_from;
  P->nb = 0;
  P->nf = 1;
  P->f_lo[0] = 0;
  P->f_hi[0] = n;
  P->shard = surfk::ceil_div(surfk::ceil_div(n, P->world), 8) * 8;   // 32-byte aligned shard starts
  for (int q = 0; q < P->world; ++q) {
    P->grad_peer[q] = static_cast<float*>(grad_peers[q]);
    P->p_peer[q] = static_cast<float*>(p_peers[q]);
    P->p16_peer[q] = static_cast<uint16_t*>(p16_peers[q]);
    if ((reinterpret_cast<uintptr_t>(grad_peers[q]) | reinterpret_cast<uintptr_t>(p_peers[q])) & 15u)
      return static_cast<int>(cudaErrorMisalignedAddress);
    if (reinterpret_cast<uintptr_t>(p16_peers[q]) & 7u) return static_cast<int>(cudaErrorMisalignedAddress);
  }
  P->m = m;
  P->v = v;
  P->hyper = hyper;
  if ((reinterpret_cast<uintptr_t>(m) | reinterpret_cast<uintptr_t>(v)) & 15u)
    return static_cast<int>(cudaErrorMisalignedAddress);
  return 0;
}

SURF_EXPORT int64_t surf_p2p_shard(void* plan) { return static_cast<Plan*>(plan)->shard; }

// Every rank's bf16 gradient copy (n elements each, 16-byte aligned): the
// buffer the peers read. Required before the first step.
SURF_EXPORT int surf_p2p_set_grad16(void* plan, void* const* g16_peers) {
  Plan* P = static_cast<Plan*>(plan);
  for (int q = 0; q < P->world; ++q) {
    P->g16_peer[q] = static_cast<uint16_t*>(g16_peers[q]);
    if (!g16_peers[q] || (reinterpret_cast<uintptr_t>(g16_peers[q]) & 15u))
      return static_cast<int>(cudaErrorMisalignedAddress);
  }
  return 0;
}

// Overlapped buckets: nb (<= 2) sorted, disjoint ranges [lo, hi) of the
// gradient, boundaries multiples of 8; the step kernel reduces the rest.
// nb = 0: the step kernel reduces everything.
SURF_EXPORT int surf_p2p_set_buckets(void* plan, int nb, const int64_t* lo, const int64_t* hi) {
  Plan* P = static_cast<Plan*>(plan);
  if (nb < 0 || nb > kMaxB || !P->n || (P->n & 7)) return static_cast<int>(cudaErrorInvalidValue);
  int64_t prev = 0;
  for (int b = 0; b < nb; ++b)
    if (lo[b] < prev || hi[b] <= lo[b] || hi[b] > P->n || (lo[b] & 7) || (hi[b] & 7))
      return static_cast<int>(cudaErrorInvalidValue);
    else
      prev = hi[b];
  P->nb = nb;
  P->nf = 0;
  int64_t at = 0;
  for (int b = 0; b < nb; ++b) {
    P->b_lo[b] = lo[b];
    P->b_hi[b] = hi[b];
    if (lo[b] > at) { P->f_lo[P->nf] = at; P->f_hi[P->nf] = lo[b]; ++P->nf; }
    at = hi[b];
  }
  if (at < P->n) { P->f_lo[P->nf] = at; P->f_hi[P->nf] = P->n; ++P->nf; }
  return 0;
}

// Bucket b is final in this stream's order: publish its bf16 copy, release
// it to the peers, and reduce my shard's part of it (three launches).
SURF_EXPORT int surf_p2p_bucket(void* plan, int b, void* stream) {
  const Plan& P = *static_cast<const Plan*>(plan);
  if (b < 0 || b >= P.nb || !P.g16_peer[P.rank]) return static_cast<int>(cudaErrorInvalidValue);
  auto s = static_cast<cudaStream_t>(stream);
  bucket_publish_kernel<<<P.bgrid, 128, 0, s>>>(P, b);
  bucket_flag_kernel<<<1, 32, 0, s>>>(P, b);
  bucket_kernel_for(P.world)<<<P.bgrid, kBucketThreads, 0, s>>>(P, b);
  SURF_RETURN_LAUNCH();
}

SURF_EXPORT int surf_p2p_set_counts(void* plan, int64_t n, int* counts, void* const* delta_peers) {
  Plan* P = static_cast<Plan*>(plan);
  P->cn = n;
  P->counts = counts;
  for (int q = 0; q < P->world; ++q) {
    P->delta_peer[q] = static_cast<int*>(delta_peers[q]);
    if (reinterpret_cast<uintptr_t>(delta_peers[q]) & 15u) return static_cast<int>(cudaErrorMisalignedAddress);
  }
  return reinterpret_cast<uintptr_t>(counts) & 15u ? static_cast<int>(cudaErrorMisalignedAddress) : 0;
}

SURF_EXPORT int surf_p2p_grad_step(void* plan, void* stream) {
  const Plan& P = *static_cast<const Plan*>(plan);
  if (!P.n || !P.g16_peer[P.rank]) return static_cast<int>(cudaErrorInvalidValue);
  return launch_coop(grad_kernel_for(P.world), P.coop_grid, static_cast<cudaStream_t>(stream), P);
}

// Phase timestamps (ns, %globaltimer) of this rank's last gradient step:
// start, peers ready, reduce-scatter done, norms in, parameters pushed, done in.
SURF_EXPORT int surf_p2p_prof_words() { return 6; }

SURF_EXPORT int surf_p2p_moments(void* plan, double* mom, int cnt, void* stream) {
  const Plan& P = *static_cast<const Plan*>(plan);
  if (cnt < 1 || cnt > kMaxMom) return static_cast<int>(cudaErrorInvalidValue);
  moments_kernel<<<1, 256, 0, static_cast<cudaStream_t>(stream)>>>(P, mom, cnt);
  SURF_RETURN_LAUNCH();
}

SURF_EXPORT int surf_p2p_merge_counts(void* plan, void* stream) {
  const Plan& P = *static_cast<const Plan*>(plan);
  if (!P.cn) return static_cast<int>(cudaErrorInvalidValue);
  return launch_coop(counts_merge_kernel, P.coop_grid, static_cast<cudaStream_t>(stream), P);
}
