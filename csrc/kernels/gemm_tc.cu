// gemm_tc.cu — bf16 GEMM on Blackwell 5th-generation tensor cores (sm_100a).
//
//   D[M, N] = A[M, K] * B[N, K]^T      (fp32 accumulation in tensor memory)
//
// Each operand is read either K-major (row-major [rows, K]) or MN-major
// (row-major [K, rows]); the MN-major form is what lets the backward pass
// (dX = dY W, dW = dY^T X) run on the forward activations without a
// transpose. The kernel is persistent (grid = SMs x resident CTAs, static
// round-robin over 128 x BN output tiles and K splits) with 6 warps:
//
//   warp 0, one thread : TMA producer — cp.async.bulk.tensor 2-D tiles (128 B
//                        swizzle, no multicast) into a STAGES-deep smem ring
//                        shared by consecutive tiles, per-stage mbarriers;
//   warp 1, one thread : tcgen05.mma issuer — 4 MMAs (K = 16 each) per 64-wide
//                        k-tile into one of two TMEM accumulators;
//                        tcgen05.commit releases each smem stage and signals
//                        the epilogue when a tile's accumulator is complete;
//   warps 2-9          : epilogue — two warps per 32-lane TMEM quadrant, each
//                        taking every other 32-column chunk: tcgen05.ld of the
//                        warp's 32 TMEM lanes,
//                        fused bias / activation / activation-derivative,
//                        stores as fp32 or bf16, optionally also transposed,
//                        or fp32 atomic accumulation for split-K; then hand
//                        the accumulator back, so tile i's epilogue overlaps
//                        tile i+1's loads and MMAs.
//
// Every wait on an mbarrier is bounded by %globaltimer (2 s); on expiry the
// kernel records an error code in a device flag, skips the remaining work,
// releases its tensor memory and returns, so a fault in the pipeline shows
// up as an error status on the host instead of a hung GPU. Before leaving,
// the producer waits (bounded) for the loads it issued that nobody consumed
// and the MMA thread commits and waits (bounded) for its last MMAs, so no
// copy lands in released shared memory and no MMA writes freed tensor
// memory; the remaining risk is a copy or MMA that outlives those bounds.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>

#include "surf_cuda.cuh"

#include "tc_sm100.cuh"

namespace {

constexpr int kEpiWarps = 8;                   // epilogue warps (2 per TMEM lane quadrant)
constexpr int kThreads = 64 + 32 * kEpiWarps;  // producer warp + MMA warp + epilogue


// Implicit-GEMM convolution operands. An operand with mode != 0 is read
// through a 4-D tensor map over an NHWC activation (dims C, W, H, B; the map's
// element strides implement the convolution stride) instead of a 2-D matrix:
//   mode 1 (K-major, forward / input-gradient A): the 128 rows of an M tile
//          are a tw x th x tb box of output-grid positions; k-block kb is
//          tap kb / per_tap (kh = tap / kw_n, kw = tap % kw_n), channel
//          chunk kb % per_tap; the box starts at
//          (chunk * 64, w0 * sw + sign * kw, h0 * sh + sign * kh, b0);
//   mode 2 (MN-major, weight-gradient operands): the 64 rows of a k-block are
//          a tw x th x tb box of output positions (k-block = position tile),
//          the MN coordinate picks the channels: for A the output channel
//          chunk (m0), for B the tap of each 64-wide n sub-block;
//   mode 3 (16-channel activations, e.g. a depth image in 4x4 space-to-depth
//          order): one tap is 16 channels = 32 bytes, so a tap is loaded as
//          a slab of 32-byte rows with the 32-byte swizzle. A (K-major,
//          forward): k-block kb is taps 4 kb .. 4 kb + 3, one 128 x 32 B slab
//          each, and the MMA's 16-wide k step is exactly one slab. B (MN-major,
//          weight gradient): n sub-block j of 16 columns is tap n0 / 16 + j,
//          a 64 x 32 B slab of the k-block's positions; one MMA spans the
//          BN / 16 slabs (leading byte offset = slab size);
//   mode 4 (16-channel activations read as windows of two neighbouring
//          positions): the map's W stride is one position (32 B) while its
//          inner extent is two (64 B), so a box row holds taps (kw, kw + 1)
//          and is loaded with the 64-byte swizzle; window wi is (kh = wi /
//          kw_n, kw = 2 (wi % kw_n)) with kw_n = windows per kernel row.
//          A (K-major, forward): k-block kb is windows 2 kb and 2 kb + 1,
//          one 128 x 64 B box each, two MMA k steps per box. B (MN-major,
//          weight gradient): n sub-block j of 32 columns is window n0 / 32
//          + j, a 64 x 64 B box of the k-block's positions. Half the box
//          rows of mode 3 for the same bytes.
// Out-of-range coordinates (negative ones included) load zeros, which is
// what makes the padded tile edges and the transposed-convolution halo free.
struct Geo {
  int mode;
  int tw, th, tb;          // box extent in output-grid units (tw * th * tb = rows of the tile)
  int tiles_w, tiles_h;    // tiles along w / h of the output grid
  int sw, sh;              // input coordinate per output unit (the conv stride)
  int kw_n;                // taps along w
  int sign;                // +1: input = output * stride + tap; -1: input = output - tap
  int per_tap;             // 64-channel chunks per tap (mode 1)
};
// Convolution-grid output: row r of an M tile is position (b, h, w) of the
// same box decomposition as geometry A; it is stored at
// ((b * out_h + h * ys + yo) * out_w + w * xs + xo) * ldc when h < gh, w < gw
// and b < gb (the input-gradient parity classes use ys = xs = 2).
// With cls_cols > 0 the N columns are (ys * xs) parity classes of cls_cols
// channels each: class (py, px) = column / cls_cols goes to input position
// (h * ys + py, w * xs + px) — the whole stride-s input gradient in one GEMM,
// whose A operand (the output gradient) is the same for every class.
struct OutGeo {
  int on;
  int gw, gh, gb;
  int out_w, out_h, ys, xs, yo, xo;
  int cls_cols;
};
struct ConvCfg { Geo a, b; OutGeo o; };

__device__ __forceinline__ void tile_origin(const Geo& g, int t, int* b0, int* h0, int* w0) {
  const int wt = t % g.tiles_w;
  const int r = t / g.tiles_w;
  *w0 = wt * g.tw;
  *h0 = (r % g.tiles_h) * g.th;
  *b0 = (r / g.tiles_h) * g.tb;
}

template <int BN, bool A_MN, bool B_MN, int STAGES, bool RB>
struct Cfg {
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
  // RB (resident B): the whole B operand (one N tile, every k-block) is
  // loaded once per CTA and stays in shared memory; the stage ring then
  // carries A only. For the convolutions' weight operands (at most 72 KB)
  // this removes a third of the per-tile L2-to-SM traffic and half of the
  // TMA instructions.
  static constexpr int kStageBytes = RB ? kABytes : kABytes + kBBytes;
  static constexpr int kResBytes = RB ? (BN <= 32 ? 8192 : 73728) : 0;
  static constexpr int kAcc = BN <= 32 ? 8 : (BN <= 64 ? 4 : 2);   // accumulator buffers in TMEM
  static constexpr int kTmemCols = kAcc * BN;
  // epilogue warps per tile: with one 32-column chunk per tile (BN = 32) the
  // two warps of a TMEM lane quadrant take alternate tiles instead of
  // alternate chunks, so all eight epilogue warps stay busy
  static constexpr int kEpiPerTile = BN == 32 ? kEpiWarps / 2 : kEpiWarps;
  // per epilogue warp: two 32x32 fp32 staging tiles for TMA stores (4 KB
  // each); the resident-B instantiation serves convolution-grid outputs,
  // which are stored from registers, and spends that room on stages
  static constexpr int kStageOutBytes = RB ? 0 : kEpiWarps * 2 * 4096;
  // alignment slack + operand stages + barrier block (1 KB) + output staging
  static constexpr size_t kSmem =
      1024 + STAGES * static_cast<size_t>(kStageBytes) + kResBytes + 1024 + kStageOutBytes;
  // instruction descriptor: D fp32, A/B bf16, majorness, N >> 3, M >> 4
  static constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((A_MN ? 1u : 0u) << 15) |
                                     ((B_MN ? 1u : 0u) << 16) | (static_cast<uint32_t>(BN >> 3) << 17) |
                                     (static_cast<uint32_t>(BM >> 4) << 24);
};

struct Sched {             // static persistent schedule over (m block, n block, k split)
  int mt, nt, splits, per, kt_total, group;
  // Grouped rasterisation: runs of `group` m blocks sweep all n blocks, so the
  // CTAs of one wave share A and B tiles through L2.
  __device__ void tile(int t, int* m0, int* n0, int* kt0, int* nkt) const {
    const int per_split = mt * nt;
    const int sp = t / per_split;
    const int r = t - sp * per_split;
    const int span = group * nt;
    const int g = r / span;
    const int first = g * group;
    const int gsz = min(group, mt - first);
    const int local = r - g * span;
    const int mb = first + local % gsz;
    const int nb = local / gsz;
    *m0 = mb * BM;
    *n0 = nb;
    *kt0 = sp * per;
    *nkt = min(kt_total, *kt0 + per) - *kt0;
  }
  __device__ int count() const { return mt * nt * splits; }
};

// Persistent warp-specialised kernel: 10 warps = producer, MMA, 8 epilogue.
template <int BN, bool A_MN, bool B_MN, int STAGES, bool RB>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                const __grid_constant__ CUtensorMap tma_c, int use_tma_c, int M, int N, Sched sc, Epilogue ep,
                const ConvCfg cc) {
  using C = Cfg<BN, A_MN, B_MN, STAGES, RB>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tiles = smem;
  uint8_t* b_res = smem + STAGES * C::kStageBytes;      // resident B (RB), k-block kb at kb * kBBytes
  uint64_t* bars = reinterpret_cast<uint64_t*>(b_res + C::kResBytes);
  // bars: [0,S) full, [S,2S) empty, then kAcc accumulator-full, kAcc
  // accumulator-empty and the resident-B barrier
  uint64_t* acc_full = bars + 2 * STAGES;
  uint64_t* acc_empty = bars + 2 * STAGES + C::kAcc;
  uint64_t* bres_full = bars + 2 * STAGES + 2 * C::kAcc;
  uint64_t* drain = bres_full + 1;                      // the MMA thread's final commit
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  // output staging after the barrier block, 1024-aligned (swizzle atoms)
  uint8_t* stage_out = b_res + C::kResBytes + 1024;
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&bars[s]), 1);
      mbar_init(smem_u32(&bars[STAGES + s]), 1);
    }
    for (int b = 0; b < C::kAcc; ++b) {
      mbar_init(smem_u32(&acc_full[b]), 1);
      mbar_init(smem_u32(&acc_empty[b]), C::kEpiPerTile);     // one arrival per epilogue warp of the tile
    }
    mbar_init(smem_u32(bres_full), 1);
    mbar_init(smem_u32(drain), 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(C::kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;
  const int ntiles = sc.count();
  pdl_wait();          // the previous kernel's outputs (this kernel's inputs) are visible from here on
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer
      if (RB && static_cast<int>(blockIdx.x) < ntiles) {
        // the whole B operand (one N tile: n0 = 0, every k-block) once per CTA
        const uint32_t rb = smem_u32(bres_full);
        mbar_expect_tx(rb, sc.kt_total * C::kBBytes);
        for (int kb = 0; kb < sc.kt_total; ++kb) tma_load_2d(smem_u32(b_res + kb * C::kBBytes), &tma_b, kb * BK, 0, rb);
      }
      int it = 0;
      for (int t = blockIdx.x; t < ntiles && !*abort; t += gridDim.x) {
        int m0, nb, kt0, nkt;
        sc.tile(t, &m0, &nb, &kt0, &nkt);
        const int n0 = nb * BN;
        for (int i = 0; i < nkt; ++i, ++it) {
          const int s = it % STAGES;
          if (it >= STAGES && !mbar_wait(smem_u32(&bars[STAGES + s]), ((it / STAGES) & 1) ^ 1, ep.err, 1, abort)) break;
          if (ep.trace && blockIdx.x == 0 && it < kTraceN) ep.trace[it] = globaltimer();
          const uint32_t full = smem_u32(&bars[s]);
          // an MN-major A is loaded as two 64-row halves; with M <= m0 + 64
          // the second half is out of range: skip it (its stale smem rows
          // only reach accumulator rows >= M, which the epilogue drops)
          const bool a_half = (cc.a.mode == 2 || (A_MN && cc.a.mode == 0)) && m0 + 64 >= M;
          mbar_expect_tx(full, C::kStageBytes - (a_half ? BK * 128 : 0));
          const uint32_t a_dst = smem_u32(tiles + s * C::kStageBytes);
          const uint32_t b_dst = a_dst + C::kABytes;
          const int kb = kt0 + i;
          const int k = kb * BK;
          if (cc.a.mode == 1) {
            int b0, h0, w0;
            tile_origin(cc.a, m0 / BM, &b0, &h0, &w0);
            const int tap = kb / cc.a.per_tap, ch = (kb - tap * cc.a.per_tap) * 64;
            const int kh = tap / cc.a.kw_n, kw = tap - kh * cc.a.kw_n;
            tma_load_4d(a_dst, &tma_a, ch, w0 * cc.a.sw + cc.a.sign * kw, h0 * cc.a.sh + cc.a.sign * kh, b0, full);
          } else if (cc.a.mode == 2) {
            int b0, h0, w0;
            tile_origin(cc.a, kb, &b0, &h0, &w0);
            tma_load_4d(a_dst, &tma_a, m0, w0, h0, b0, full);
            if (!a_half) tma_load_4d(a_dst + BK * 128, &tma_a, m0 + 64, w0, h0, b0, full);
          } else if (cc.a.mode == 4) {
            int b0, h0, w0;
            tile_origin(cc.a, m0 / BM, &b0, &h0, &w0);
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const int wi = 2 * kb + j;
              const int kh = wi / cc.a.kw_n, kw = 2 * (wi - kh * cc.a.kw_n);
              tma_load_4d(a_dst + j * (BM * 64), &tma_a, 0, w0 * cc.a.sw + kw, h0 * cc.a.sh + kh, b0, full);
            }
          } else if (cc.a.mode == 3) {
            int b0, h0, w0;
            tile_origin(cc.a, m0 / BM, &b0, &h0, &w0);
#pragma unroll
            for (int j = 0; j < BK / 16; ++j) {
              const int tap = kb * (BK / 16) + j;
              const int kh = tap / cc.a.kw_n, kw = tap - kh * cc.a.kw_n;
              tma_load_4d(a_dst + j * (BM * 32), &tma_a, 0, w0 * cc.a.sw + kw, h0 * cc.a.sh + kh, b0, full);
            }
          } else if (A_MN) {
            tma_load_2d(a_dst, &tma_a, m0, k, full);
            if (!a_half) tma_load_2d(a_dst + BK * 128, &tma_a, m0 + 64, k, full);
          } else {
            tma_load_2d(a_dst, &tma_a, k, m0, full);
          }
          if (RB) {
            // B is resident
          } else if (cc.b.mode == 4) {
            int b0, h0, w0;
            tile_origin(cc.b, kb, &b0, &h0, &w0);
#pragma unroll 1
            for (int j = 0; j < BN / 32; ++j) {
              const int wi = n0 / 32 + j;
              const int kh = wi / cc.b.kw_n, kw = 2 * (wi - kh * cc.b.kw_n);
              tma_load_4d(b_dst + j * (BK * 64), &tma_b, 0, w0 * cc.b.sw + kw, h0 * cc.b.sh + kh, b0, full);
            }
          } else if (cc.b.mode == 3) {
            int b0, h0, w0;
            tile_origin(cc.b, kb, &b0, &h0, &w0);
#pragma unroll 1
            for (int j = 0; j < BN / 16; ++j) {
              const int tap = n0 / 16 + j;
              const int kh = tap / cc.b.kw_n, kw = tap - kh * cc.b.kw_n;
              tma_load_4d(b_dst + j * (BK * 32), &tma_b, 0, w0 * cc.b.sw + kw, h0 * cc.b.sh + kh, b0, full);
            }
          } else if (cc.b.mode == 2) {
            int b0, h0, w0;
            tile_origin(cc.b, kb, &b0, &h0, &w0);
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) {
              const int tap = n0 / 64 + j;
              const int kh = tap / cc.b.kw_n, kw = tap - kh * cc.b.kw_n;
              tma_load_4d(b_dst + j * BK * 128, &tma_b, 0, w0 * cc.b.sw + kw, h0 * cc.b.sh + kh, b0, full);
            }
          } else if (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(b_dst + j * BK * 128, &tma_b, n0 + 64 * j, k, full);
          } else {
            tma_load_2d(b_dst, &tma_b, k, n0, full);
          }
        }
      }
      if (*abort) {
        // loads may still be landing in stages nobody consumes: wait for them
        // (bounded) before the CTA's shared memory goes away
        for (int j = it > STAGES ? it - STAGES : 0; j < it; ++j)
          mbar_wait_bounded(smem_u32(&bars[j % STAGES]), (j / STAGES) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer
      int it = 0, tc = 0;
      bool res_ok = true;
      if (RB && static_cast<int>(blockIdx.x) < ntiles) {
        res_ok = mbar_wait(smem_u32(bres_full), 0, ep.err, 5, abort);
        fence_after();
      }
      // UMMA descriptors: the layout / LBO / SBO bits and every k step's start
      // offset are fixed for the launch; per stage only the base address
      // (the low 14-bit field, in 16-byte units) is added.
      // K-major: +32 B per 16-element k step inside the 128 B swizzled row;
      // MN-major: +2 k-groups (2 x 1024 B) per step; MN blocks BK*128 B apart.
      // Mode 3 (32 B swizzle): A steps one 128-row slab per k step (8-row
      // groups 256 B apart); B steps 16 positions (512 B) inside every
      // 16-column slab, the slabs BK*32 B apart.
      // Mode 4 (64 B swizzle): A k steps 0-1 lie in window box 0 and
      // 2-3 in box 1 (+32 B per step inside a 64 B row, 8-row groups
      // 512 B apart); B steps 16 positions (1024 B) inside every
      // 32-column window box, the boxes BK*64 B apart.
      const uint64_t a_proto = cc.a.mode == 3   ? smem_desc(0, 16, 256, kSw32)
                               : cc.a.mode == 4 ? smem_desc(0, 16, 512, kSw64)
                               : A_MN           ? smem_desc(0, BK * 128, 1024)
                                                : smem_desc(0, 16, 1024);
      const uint64_t b_proto = cc.b.mode == 3   ? smem_desc(0, BK * 32, 256, kSw32)
                               : cc.b.mode == 4 ? smem_desc(0, BK * 64, 512, kSw64)
                               : B_MN           ? smem_desc(0, BK * 128, 1024)
                                                : smem_desc(0, 16, 1024);
      uint32_t a_step[BK / 16], b_step[BK / 16];
#pragma unroll
      for (int j = 0; j < BK / 16; ++j) {
        a_step[j] = (cc.a.mode == 3 ? j * (BM * 32) : cc.a.mode == 4 ? (j >> 1) * (BM * 64) + (j & 1) * 32
                     : A_MN ? j * 2048 : j * 32) >> 4;
        b_step[j] = (cc.b.mode == 3 ? j * 512 : cc.b.mode == 4 ? j * 1024 : B_MN ? j * 2048 : j * 32) >> 4;
      }
      for (int t = blockIdx.x; res_ok && t < ntiles && !*abort; t += gridDim.x, ++tc) {
        int m0, nb, kt0, nkt;
        sc.tile(t, &m0, &nb, &kt0, &nkt);
        const int buf = tc % C::kAcc, use = tc / C::kAcc;
        if (use > 0 && !mbar_wait(smem_u32(&acc_empty[buf]), (use & 1) ^ 1, ep.err, 4, abort)) break;
        fence_after();
        const uint32_t dtm = tmem + buf * BN;
        bool ok = true;
        for (int i = 0; i < nkt; ++i, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(smem_u32(&bars[s]), (it / STAGES) & 1, ep.err, 2, abort)) { ok = false; break; }
          fence_after();
          if (ep.trace && blockIdx.x == 0 && it < kTraceN) ep.trace[kTraceN + it] = globaltimer();
          const uint32_t a_base = smem_u32(tiles + s * C::kStageBytes);
          const uint32_t b_base = RB ? smem_u32(b_res + (kt0 + i) * C::kBBytes) : a_base + C::kABytes;
          const uint64_t da0 = a_proto + (a_base >> 4), db0 = b_proto + (b_base >> 4);
          if (!(ep.dbg & 2)) {
#pragma unroll
            for (int j = 0; j < BK / 16; ++j)
              mma_bf16(dtm, da0 + a_step[j], db0 + b_step[j], C::kIdesc, (i > 0 || j > 0) ? 1u : 0u);
          }
          mma_commit(smem_u32(&bars[STAGES + s]));      // frees the stage when these MMAs finish
          if (ep.trace && blockIdx.x == 0 && it < kTraceN) ep.trace[2 * kTraceN + it] = globaltimer();
        }
        if (!ok) break;
        mma_commit(smem_u32(&acc_full[buf]));          // accumulator of this tile complete
      }
      // every MMA issued by this thread has completed before the tensor memory is freed
      mma_commit(smem_u32(drain));
      mbar_wait_bounded(smem_u32(drain), 0);
    }
  } else {
    // ---- epilogue warps 2..9 (TMEM lane quadrant = warp % 4; `half` picks
    // the even or odd 32-column chunks of the tile)
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    int tc = 0;
    int stage_ctr = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++tc) {
      int m0, nb, kt0, nkt;
      sc.tile(t, &m0, &nb, &kt0, &nkt);
      const int n0 = nb * BN;
      const int buf = tc % C::kAcc, use = tc / C::kAcc;
      if (BN == 32 && (tc & 1) != half) continue;      // the other warp of this quadrant takes the tile
      int row = m0 + quad * 32 + lane;
      bool row_ok = row < M;
      int64_t roff = static_cast<int64_t>(row);         // row index in units of ldc / ld_aux
      int gpos_b = 0, gpos_h = 0, gpos_w = 0;
      if (cc.o.on) {
        int b0, h0, w0;
        tile_origin(cc.a, m0 / BM, &b0, &h0, &w0);
        const int r = quad * 32 + lane;
        const int wi = r % cc.a.tw, hi = (r / cc.a.tw) % cc.a.th, bi = r / (cc.a.tw * cc.a.th);
        gpos_w = w0 + wi;
        gpos_h = h0 + hi;
        gpos_b = b0 + bi;
        row_ok = gpos_w < cc.o.gw && gpos_h < cc.o.gh && gpos_b < cc.o.gb;
        roff = (static_cast<int64_t>(gpos_b) * cc.o.out_h + gpos_h * cc.o.ys + cc.o.yo) * cc.o.out_w +
               gpos_w * cc.o.xs + cc.o.xo;
      }
      // where this lane's row of the 32-column chunk at tile column c0 goes:
      // output row, validity, first column and columns per row (a parity
      // class of a strided input gradient has its own rows)
      auto chunk_loc = [&](int c0, int64_t& off, bool& ok, int& col, int& ncol) {
        if (cc.o.cls_cols) {
          const int cls = (n0 + c0) / cc.o.cls_cols;
          col = n0 + c0 - cls * cc.o.cls_cols;
          const int hh = gpos_h * cc.o.ys + cls / cc.o.xs, ww = gpos_w * cc.o.xs + cls % cc.o.xs;
          ok = row_ok && hh < cc.o.out_h && ww < cc.o.out_w;
          off = (static_cast<int64_t>(gpos_b) * cc.o.out_h + hh) * cc.o.out_w + ww;
          ncol = cc.o.cls_cols;
        } else {
          off = roff;
          ok = row_ok;
          col = n0 + c0;
          ncol = N;
        }
      };
      // the derivative modes read the saved activation of each output row:
      // the first chunk's is loaded before the accumulator is waited for,
      // each next chunk's while the current one is stored
      const int c_first = BN == 32 ? 0 : 32 * half;
      uint4 pre[4];
      bool have = false;
      auto prefetch = [&](int c0) {
        have = false;
        if (c0 < BN && n0 + c0 < N && !(ep.dbg & 8)) {
          int64_t off;
          bool ok;
          int col, ncol;
          chunk_loc(c0, off, ok, col, ncol);
          have = load_aux32(ep, off, ok, col, ncol, pre);
        }
      };
      if (!(ep.dbg & 1)) prefetch(c_first);
      if (!mbar_wait(smem_u32(&acc_full[buf]), use & 1, ep.err, 3, abort)) break;
      fence_after();
      if (ep.trace && blockIdx.x == 0 && warp == 2 && lane == 0 && tc < kTraceN) ep.trace[3 * kTraceN + tc] = globaltimer();
      if (ep.dbg & 1) {
        float v[32];
        tmem_ld32(tmem + (static_cast<uint32_t>(quad * 32) << 16) + buf * BN, v);
        if (v[0] == 12345.0f && row < 0) ep.err[0] = 1;      // keep the load alive
      } else if (use_tma_c) {
        // bias/activation in registers, then the warp's 32 x 32 chunk goes to a
        // swizzled smem tile and out with one asynchronous TMA store
        const bool bf = ep.c_dtype == 1;
        uint8_t* my_stage = stage_out + (warp - 2) * 8192;
#pragma unroll 1
        for (int c0 = c_first; c0 < BN; c0 += 64) {
          if (n0 + c0 >= N) break;
          float v[32];
          tmem_ld32(tmem + (static_cast<uint32_t>(quad * 32) << 16) + buf * BN + c0, v);
          process_chunk32(ep, v, roff, row_ok, n0 + c0, N, have ? pre : nullptr);
          prefetch(c0 + 64);
          const int sb = stage_ctr & 1;
          if (lane == 0 && stage_ctr >= 2) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
          __syncwarp();
          uint8_t* tile = my_stage + sb * 4096;
          if (bf) {
            // 64-byte rows, 64 B swizzle: 16 B chunk c of row r lands at chunk c ^ ((r >> 1) & 3)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              uint32_t w[4];
#pragma unroll
              for (int k = 0; k < 4; ++k)
                w[k] = surfk::pack_bf16x2(v[8 * c + 2 * k], v[8 * c + 2 * k + 1]);
              const int pc = c ^ ((lane >> 1) & 3);
              *reinterpret_cast<uint4*>(tile + lane * 64 + pc * 16) = make_uint4(w[0], w[1], w[2], w[3]);
            }
          } else {
            // 128-byte rows, 128 B swizzle: chunk c of row r lands at chunk c ^ (r & 7)
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const int pc = c ^ (lane & 7);
              *reinterpret_cast<float4*>(tile + lane * 128 + pc * 16) =
                  make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
            }
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          // a remapped output column (cmap): 32-column chunks never straddle a segment
          const int oc = ep.cmap_in ? ((n0 + c0) / ep.cmap_in) * ep.cmap_out + (n0 + c0) % ep.cmap_in : n0 + c0;
          if (lane == 0) tma_store_2d(&tma_c, smem_u32(tile), oc, m0 + quad * 32);
          ++stage_ctr;
        }
      } else {
#pragma unroll 1
        for (int c0 = c_first; c0 < BN; c0 += 64) {
          if (n0 + c0 >= N) break;
          int64_t off;
          bool ok;
          int col, ncol;
          chunk_loc(c0, off, ok, col, ncol);
          float v[32];
          tmem_ld32(tmem + (static_cast<uint32_t>(quad * 32) << 16) + buf * BN + c0, v);
          process_chunk32(ep, v, off, ok, col, ncol, have ? pre : nullptr);
          prefetch(c0 + 64);
          store_chunk32(ep, v, off, ok, col, ncol);
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&acc_empty[buf])) : "memory");
      if (ep.trace && blockIdx.x == 0 && warp == 2 && lane == 0 && tc < kTraceN) ep.trace[4 * kTraceN + tc] = globaltimer();
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::kTmemCols));
}

// ---- host side ---------------------------------------------------------------
// A 4-D bf16 NHWC activation view for an implicit-convolution operand.
struct MapDesc {
  const void* base;
  int64_t dims[4];          // C, W, H, B (elements)
  int64_t strides[3];       // bytes between consecutive W, H, B positions (multiples of 16)
  int box[4];               // box extent per dimension, in elements (element strides included)
  int estr[4];              // element (traversal) strides
};

bool make_map4d(CUtensorMap* m, const MapDesc& d) {
  auto fn = encode_fn();
  if (!fn) return false;
  const int inner = d.box[0] * 2;     // bytes: the swizzle span follows the box's inner extent
  if ((reinterpret_cast<uintptr_t>(d.base) & 15) || (inner != 32 && inner != 64 && inner != 128)) return false;
  const CUtensorMapSwizzle swz = inner == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                 : inner == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
  cuuint64_t dims[4], strides[3];
  cuuint32_t box[4], estr[4];
  for (int i = 0; i < 4; ++i) {
    dims[i] = static_cast<cuuint64_t>(d.dims[i]);
    box[i] = static_cast<cuuint32_t>(d.box[i]);
    estr[i] = static_cast<cuuint32_t>(d.estr[i]);
    if (d.box[i] < 1 || d.box[i] > 256 || d.estr[i] < 1 || d.estr[i] > 8) return false;
  }
  for (int i = 0; i < 3; ++i) {
    strides[i] = static_cast<cuuint64_t>(d.strides[i]);
    if (d.strides[i] % 16) return false;
  }
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(d.base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int BN, bool A_MN, bool B_MN, int STAGES, bool RB>
int launch_cfg(const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N, int K, const Epilogue& ep,
               int splits, cudaStream_t s, const MapDesc* ad, const MapDesc* bd, const ConvCfg& cc) {
  using C = Cfg<BN, A_MN, B_MN, STAGES, RB>;
  static_assert(C::kSmem <= 232448, "shared memory per CTA");
  auto kern = gemm_kernel<BN, A_MN, B_MN, STAGES, RB>;
  CUtensorMap ta, tb;
  const bool okA = ad ? make_map4d(&ta, *ad)
                      : (A_MN ? make_map(&ta, A, M, K, lda, 64, BK) : make_map(&ta, A, K, M, lda, BK, BM));
  const bool okB = bd ? make_map4d(&tb, *bd)
                      : (B_MN ? make_map(&tb, B, N, K, ldb, 64, BK) : make_map(&tb, B, K, N, ldb, BK, BN));
  if (!okA || !okB) return static_cast<int>(cudaErrorInvalidValue);
  // TMA-store epilogue for plain stores with 16-byte aligned rows
  CUtensorMap tc;
  std::memset(&tc, 0, sizeof tc);
  const int esize = ep.c_dtype == 1 ? 2 : 4;
  // (a column remap keeps the TMA store when every chunk is whole: N % 32 == 0)
  const int c_cols = ep.cmap_in ? (N / ep.cmap_in) * ep.cmap_out + N % ep.cmap_in : N;
  int use_tma_c = ep.c && ep.c_mode == kStore && !ep.ct && !cc.o.on && (!ep.cmap_in || N % 32 == 0) &&
                  ((reinterpret_cast<uintptr_t>(ep.c) & 15) == 0) && ((ep.ldc * esize) % 16 == 0);
  if (use_tma_c)
    use_tma_c = make_map(&tc, ep.c, c_cols, M, ep.ldc, 32, 32, ep.c_dtype != 1,
                         ep.c_dtype == 1 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B)
                    ? 1
                    : 0;
  const cudaError_t attr = smem_limit_once<gemm_kernel<BN, A_MN, B_MN, STAGES, RB>>(static_cast<int>(C::kSmem));
  if (attr != cudaSuccess) return static_cast<int>(attr);
  static int resident = 0;          // CTAs per SM for this instantiation
  static int sms = 0;
  if (!resident) {
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, kern, kThreads, C::kSmem);
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (resident < 1) resident = 1;
    if (resident * C::kTmemCols > 512) resident = 512 / C::kTmemCols;
  }
  Sched sc;
  sc.kt_total = (K + BK - 1) / BK;
  if (splits < 1) splits = 1;
  if (splits > sc.kt_total) splits = sc.kt_total;
  sc.per = (sc.kt_total + splits - 1) / splits;
  sc.splits = (sc.kt_total + sc.per - 1) / sc.per;
  sc.mt = (M + BM - 1) / BM;
  sc.nt = (N + BN - 1) / BN;
  sc.group = 8;
  const int64_t ntiles = static_cast<int64_t>(sc.mt) * sc.nt * sc.splits;
  const int grid = static_cast<int>(ntiles < static_cast<int64_t>(sms) * resident ? ntiles : static_cast<int64_t>(sms) * resident);
  launch_pdl(kern, dim3(grid), dim3(kThreads), C::kSmem, s, ta, tb, tc, use_tma_c, M, N, sc, ep, cc);
  SURF_RETURN_LAUNCH();
}

template <int BN, bool A_MN, bool B_MN>
int launch(const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N, int K, const Epilogue& ep, int splits,
           cudaStream_t s, const MapDesc* ad = nullptr, const MapDesc* bd = nullptr, const ConvCfg* conv = nullptr) {
  // as many stages as fit next to the output staging (227 KB per CTA): the
  // implicit convolutions re-read every input tile once per tap from L2, so
  // their throughput is bytes in flight / latency
  constexpr int STAGES = BN <= 32 ? 8 : (BN <= 64 ? 6 : (BN <= 128 ? 5 : 3));
  ConvCfg cc;
  std::memset(&cc, 0, sizeof cc);
  if (conv) cc = *conv;
  if constexpr (!A_MN && !B_MN && BN <= 64) {
    // implicit convolution with a K-major activation A and a plain weight B
    // of one N tile, unsplit: keep B resident (diagnostic bit 2 turns it off).
    // Measured at 4,096 images, resident against streamed in the same run:
    // conv1 forward 8% faster, conv2 / conv3 forward and the stride-1 input
    // gradient 0-11% depending on the machine; the 128-wide parity-class input
    // gradient was 4% slower and keeps streaming B. 13 / 9 stages instead of
    // 8 / 5 (the room of the unused output staging) measured the same.
    constexpr int RB_STAGES = BN <= 32 ? 13 : 9;
    using R = Cfg<BN, false, false, RB_STAGES, true>;
    const int kt = (K + BK - 1) / BK;
    if ((cc.a.mode == 1 || cc.a.mode == 3 || cc.a.mode == 4) && cc.o.on && !bd && cc.b.mode == 0 && N <= BN && splits <= 1 && kt * R::kBBytes <= R::kResBytes &&
        !(ep.dbg & 4))
      return launch_cfg<BN, false, false, RB_STAGES, true>(A, lda, B, ldb, M, N, K, ep, 1, s, ad, bd, cc);
  }
  return launch_cfg<BN, A_MN, B_MN, STAGES, false>(A, lda, B, ldb, M, N, K, ep, splits, s, ad, bd, cc);
}

template <int BN>
int dispatch_major(const void* A, int64_t lda, int a_mn, const void* B, int64_t ldb, int b_mn, int M, int N, int K,
                   const Epilogue& ep, int splits, cudaStream_t s, const MapDesc* ad = nullptr,
                   const MapDesc* bd = nullptr, const ConvCfg* cc = nullptr) {
  if (a_mn && b_mn) return launch<BN, true, true>(A, lda, B, ldb, M, N, K, ep, splits, s, ad, bd, cc);
  if (a_mn) return launch<BN, true, false>(A, lda, B, ldb, M, N, K, ep, splits, s, ad, bd, cc);
  if (b_mn) return launch<BN, false, true>(A, lda, B, ldb, M, N, K, ep, splits, s, ad, bd, cc);
  return launch<BN, false, false>(A, lda, B, ldb, M, N, K, ep, splits, s, ad, bd, cc);
}

}  // namespace

// D = A * B^T with a fused epilogue. a_mn / b_mn select MN-major operands
// (row-major [K, M] / [K, N]); otherwise operands are row-major [M, K] / [N, K].
// Leading dimensions in elements (multiples of 8). bn: tile width 32/64/128/256
// (MN-major B needs bn >= 64). splits > 1 partitions K over grid.z and
// requires the atomic fp32 output mode.
SURF_EXPORT int surf_gemm_bf16(const void* A, int64_t lda, int a_mn, const void* B, int64_t ldb, int b_mn, int M,
                               int N, int K, const Epilogue* ep, int bn, int splits, void* stream) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  if ((lda & 7) || (ldb & 7)) return static_cast<int>(cudaErrorInvalidValue);
  if (splits > 1 && ep->c_mode != kAtomic) return static_cast<int>(cudaErrorInvalidValue);
  if (b_mn && bn < 64) return static_cast<int>(cudaErrorInvalidValue);
  if (ep->act_split < N && (ep->act_split & 31)) return static_cast<int>(cudaErrorInvalidValue);
  if (ep->cmap_in && ((ep->cmap_in & 31) || ep->cmap_out < ep->cmap_in)) return static_cast<int>(cudaErrorInvalidValue);
  auto s = static_cast<cudaStream_t>(stream);
  switch (bn) {
    case 32: return dispatch_major<32>(A, lda, a_mn, B, ldb, b_mn, M, N, K, *ep, splits, s);
    case 64: return dispatch_major<64>(A, lda, a_mn, B, ldb, b_mn, M, N, K, *ep, splits, s);
    case 128: return dispatch_major<128>(A, lda, a_mn, B, ldb, b_mn, M, N, K, *ep, splits, s);
    case 256: return dispatch_major<256>(A, lda, a_mn, B, ldb, b_mn, M, N, K, *ep, splits, s);
    default: return static_cast<int>(cudaErrorInvalidValue);
  }
}

SURF_EXPORT int surf_gemm_epilogue_size() { return static_cast<int>(sizeof(Epilogue)); }

// Implicit-GEMM convolution: the same kernel with 4-D activation operands.
// ad / bd (either may be null = a plain 2-D operand with lda / ldb) describe
// NHWC activation views; cc gives the tile geometry of each operand and of a
// convolution-grid output (see Geo / OutGeo). M for a mode-1 A is the number
// of M tiles x 128; K for mode-2 operands is the number of position tiles x 64.
SURF_EXPORT int surf_gemm_conv(const void* A, int64_t lda, const MapDesc* ad, int a_mn, const void* B, int64_t ldb,
                               const MapDesc* bd, int b_mn, int M, int N, int K, const Epilogue* ep,
                               const ConvCfg* cc, int bn, int splits, void* stream) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  if (splits > 1 && ep->c_mode != kAtomic) return static_cast<int>(cudaErrorInvalidValue);
  if (b_mn && bn < 64) return static_cast<int>(cudaErrorInvalidValue);
  if ((cc->a.mode == 1 && a_mn) || (cc->a.mode == 2 && !a_mn) || ((cc->a.mode == 3 || cc->a.mode == 4) && a_mn) ||
      (cc->b.mode == 2 && !b_mn) || ((cc->b.mode == 3 || cc->b.mode == 4) && !b_mn) || cc->b.mode == 1 ||
      cc->a.mode > 4 || cc->b.mode > 4)
    return static_cast<int>(cudaErrorInvalidValue);
  if ((cc->a.mode && !ad) || (cc->b.mode && !bd)) return static_cast<int>(cudaErrorInvalidValue);
  if ((cc->a.mode == 1 || cc->a.mode == 3 || cc->a.mode == 4) && cc->a.tw * cc->a.th * cc->a.tb != BM)
    return static_cast<int>(cudaErrorInvalidValue);
  if (cc->a.mode == 2 && cc->a.tw * cc->a.th * cc->a.tb != BK) return static_cast<int>(cudaErrorInvalidValue);
  if ((cc->b.mode == 2 || cc->b.mode == 3 || cc->b.mode == 4) && cc->b.tw * cc->b.th * cc->b.tb != BK)
    return static_cast<int>(cudaErrorInvalidValue);
  // mode 3 slabs: 16-channel boxes (32-byte rows); B spans whole taps of 16 columns
  if (cc->a.mode == 3 && (!ad || ad->box[0] != 16)) return static_cast<int>(cudaErrorInvalidValue);
  if (cc->b.mode == 3 && (!bd || bd->box[0] != 16 || bn != 64)) return static_cast<int>(cudaErrorInvalidValue);
  // mode 4 windows: 32-element (64-byte) box rows, a k-block of A is two
  // windows (K = 64 per k-block), B sub-blocks are whole 32-column windows
  if (cc->a.mode == 4 && (!ad || ad->box[0] != 32 || cc->a.kw_n < 1)) return static_cast<int>(cudaErrorInvalidValue);
  if (cc->b.mode == 4 && (!bd || bd->box[0] != 32 || bn != 64 || cc->b.kw_n < 1))
    return static_cast<int>(cudaErrorInvalidValue);
  if (cc->o.on && cc->a.mode != 1 && cc->a.mode != 3 && cc->a.mode != 4) return static_cast<int>(cudaErrorInvalidValue);
  if (cc->o.cls_cols && (cc->o.cls_cols % 32 || N != cc->o.cls_cols * cc->o.ys * cc->o.xs))
    return static_cast<int>(cudaErrorInvalidValue);
  if (ep->act_split < N && (ep->act_split & 31)) return static_cast<int>(cudaErrorInvalidValue);
  auto s = static_cast<cudaStream_t>(stream);
  switch (bn) {
    case 32: return dispatch_major<32>(A, lda, a_mn, B, ldb, b_mn, M, N, K, *ep, splits, s, ad, bd, cc);
    case 64: return dispatch_major<64>(A, lda, a_mn, B, ldb, b_mn, M, N, K, *ep, splits, s, ad, bd, cc);
    case 128: return dispatch_major<128>(A, lda, a_mn, B, ldb, b_mn, M, N, K, *ep, splits, s, ad, bd, cc);
    case 256: return dispatch_major<256>(A, lda, a_mn, B, ldb, b_mn, M, N, K, *ep, splits, s, ad, bd, cc);
    default: return static_cast<int>(cudaErrorInvalidValue);
  }
}

SURF_EXPORT int surf_gemm_conv_sizes(int* out) {
  out[0] = static_cast<int>(sizeof(MapDesc));
  out[1] = static_cast<int>(sizeof(ConvCfg));
  return 0;
}
