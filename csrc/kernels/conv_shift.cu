// conv_shift.cu — convolutions as GEMMs over row-shifted views of flattened
// activation grids (sm_100a, tcgen05 + TMEM + TMA).
//
// An activation is a [rows, channels] matrix whose row p is grid position
// (b, h, w), p = (b*GH + h)*GW + w. For a stride-1 convolution computed at
// EVERY grid position (rows whose output lies outside the valid window are
// computed and dropped), the input row that tap (kh, kw) of output row p
// reads is row p + kh*GW + kw: every tap is the same matrix shifted by a
// constant number of rows. A 128-row tile of outputs needs ONE contiguous box
// of input rows, loaded by a single TMA copy, and each tap's MMA reads that
// box at its row shift. UMMA descriptors and the TMA unit both apply the
// 128-, 64- and 32-byte swizzles to absolute shared-memory address bits, so a
// descriptor may start at any row of the box (measured on a B200: every row
// offset matches a plain GEMM with base offset 0). Stride 2 is folded into
// the views: two neighbouring positions form one 2x-wide "pair" row, and the
// rows of one input-row parity form a plane read by a 3-D box (row stride 2).
//
// A tcgen05.mma of 128 x N x 16 costs about the same time for every N up to
// 256 (measured: ~141 cycles per instruction at N = 32..256), so both kinds
// fill the accumulator with useful partial sums:
//
//   FWD    (forward and input gradient) output rows = grid positions, A
//          (K-major) = the shifted input box, B = weights resident in shared
//          memory. "Row stacking": the accumulator has nblk column blocks;
//          block j at accumulator row p is the partial sum of output row
//          p - bd[j] over the taps whose shift is the instruction's shift +
//          bd[j], so one A operand feeds up to nblk taps. The epilogue adds
//          block j of row q + bd[j] (a warp shuffle) into output row q, then
//          bias + ReLU, or the ReLU derivative from the saved activation, and
//          stores bf16 through an output map (valid window, class scatter).
//          Rows q + bd[j] past the warp contribute zero: the caller's grids
//          put only invalid (or exactly zero) outputs in those lanes.
//   WGRAD  D += dY^T x shifted inputs, k = grid positions. "Position
//          stacking": A (MN-major) holds the output gradient of two position
//          ranges L rows apart (its two 64-wide MN blocks, LBO = L rows), so
//          the upper accumulator half computes the taps L rows below the
//          lower half's; B (MN-major) = the input box, MMA group g's N blocks
//          b_lbo apart from b_noff[g]. A per-(32-row, 16-column) block table
//          maps the accumulator onto the weight gradient (duplicates skipped);
//          fp32 atomics, K split over CTAs.
//
// Warps: 0 TMA producer (one thread), 1 MMA issuer (one thread), 2-9
// epilogue (two per TMEM lane quadrant). Every mbarrier wait is bounded; on
// expiry the kernel records an error code, waits for its copies in flight
// (bounded), releases its tensor memory and returns.
#include "tc_sm100.cuh"

#include <climits>

namespace {

constexpr int kShEpiWarps = 8;
constexpr int kShThreads = 64 + 32 * kShEpiWarps;
constexpr int kShMaxKSteps = 64;       // FWD: K <= 1024
constexpr int kShMaxSub = 16;          // WGRAD: MMA groups
constexpr int kShMaxStages = 8;
constexpr int kShMaxNb16 = 32;         // WGRAD: 16-column blocks of the accumulated N (<= 512)

enum ShKind : int { kShFwd = 0, kShWgrad = 1 };

struct ShSeg {         // one TMA box of a load unit (FWD: a tile; WGRAD: a k-block)
  int rows;            // box rows (grid rows)
  int row_bytes;       // 32, 64 or 128
  int gw;              // 0: 2-D box; else a 3-D box of rows / gw groups of gw rows (row coordinate / gw)
  int udiv;            // unit u -> first row (u / udiv) * mul_hi + (u % udiv) * mul_lo + add
  int mul_hi, mul_lo, add;
  int soff;            // byte offset of the box in a stage (multiple of 1024)
};

struct ShOut {         // output row p of the grid -> destination (and saved-activation) location
  int gw, gh;          // p = (b * gh + h) * gw + w
  int vh, vw;          // kept when hh < vh and ww < vw, hh = h * ys + py, ww = w * xs + px
  int ys, xs;          // class = column block: py = class / xs, px = class % xs
  int cls_cols;        // columns per class (0: no classes)
  int hp, wp;          // parity splits of hh / ww (1 or 2)
  int owc;             // column offset of ww % wp
  int64_t ob, ohp, oh, ow;   // row = b*ob + (hh % hp)*ohp + (hh / hp)*oh + (ww / wp)*ow
};

struct ShArgs {
  int kind;
  int M, N;            // FWD: M = grid rows, N = accumulator columns (nblk blocks); WGRAD: N = accumulator columns
  int kt;              // FWD: 64-wide k-blocks of the resident B; WGRAD: load units in total
  int mt;              // FWD: tiles
  int nt, splits, per; // WGRAD: N tiles, K splits, load units per split
  int nseg_a, nseg_b;  // boxes per load unit: A ones first, then B ones
  ShSeg seg[4];
  int stage_bytes;
  int unit_bytes;      // bytes one load unit lands (the full barrier's transaction count)
  int a_layout, a_lbo, a_sbo;
  int b_layout, b_lbo, b_sbo;
  int ksteps;          // FWD: 16-wide K steps per tile; WGRAD: 16-position K steps per load unit
  int a_koff[kShMaxKSteps];  // FWD: stage byte offset of K step ks's A operand (row shift + in-row offset)
  int nblk;            // FWD: accumulator column blocks (1..4) of N / nblk columns
  int bd[4];           // FWD: block j of accumulator row p belongs to output row p - bd[j] (0..2)
  int zero_fill;       // FWD: rows outside the valid window are stored as zeros (else skipped)
  int stg_bytes;       // FWD: shared-memory output block of one epilogue warp (multiple of 16)
  int a_off, a_krow;   // WGRAD: stage byte offset of A, bytes per k-row
  int subw, b_krow;    // WGRAD: N of one MMA group, bytes per k-row of B
  int b_noff[kShMaxSub];     // WGRAD: stage byte offset of MMA group g (global index n / subw)
  int kgrid, kmask;    // WGRAD: K step ks of a unit covers grid row h = (A-box row / 16 + ks) mod kgrid;
                       //   only the rows in kmask are issued (the others' output gradient is zero)
  int bias_rows;       // WGRAD: > 0: also sum the first bias_rows rows of every unit's A box (128-byte rows)
  int bias_mod;        //   into the bias gradient (Epilogue.ct, fp32): column c adds to channel c % bias_mod
  int erow[4];         // WGRAD: destination row of accumulator row m = (m & 31) + erow[m >> 5]
  short ecol[4][kShMaxNb16]; // WGRAD: destination column of 16-column block n >> 4 for rows m >> 5 (-1: skip)
  ShOut om;
};

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}

__device__ __forceinline__ int seg_row(const ShSeg& s, int u) {
  return (u / s.udiv) * s.mul_hi + (u % s.udiv) * s.mul_lo + s.add;
}

__device__ __forceinline__ const CUtensorMap* pick(int i, const CUtensorMap* m0, const CUtensorMap* m1,
                                                   const CUtensorMap* m2, const CUtensorMap* m3) {
  return i == 0 ? m0 : i == 1 ? m1 : i == 2 ? m2 : m3;
}

template <int BN, int KIND>
struct ShCfg {
  static constexpr int kAcc = BN <= 128 ? 4 : BN <= 256 ? 2 : 1;
  static constexpr int kCols = kAcc * BN;
  static constexpr int kTmemCols = kCols <= 32 ? 32 : kCols <= 64 ? 64 : kCols <= 128 ? 128 : kCols <= 256 ? 256 : 512;
  // FWD: the two epilogue halves take alternate tiles (4 warps per tile);
  // WGRAD: both halves split one unit's columns
  static constexpr int kEpiPerTile = KIND == kShFwd ? kShEpiWarps / 2 : kShEpiWarps;
};

// 16-byte asynchronous global -> shared copy (LSU path, not the TMA unit)
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

// the epilogue's shared-memory block is stored with its 16-byte chunks
// permuted inside each 128-byte line (chunk i at i ^ (line & 7)): the rows a
// warp writes are 64 or 128 bytes apart, which would otherwise put every lane
// on the same banks
__device__ __forceinline__ int stg_chunk(int i) { return i ^ ((i >> 3) & 7); }

// FWD output location of (grid position, 32-column chunk c0): destination row
// and column, and whether the position lies in the valid window
struct ShLoc {
  int64_t row;
  int dcol, col;
  bool valid;
};

__device__ __forceinline__ ShLoc sh_locate(const ShOut& o, int b, int h, int w, int c0) {
  int cls = 0, col = c0;
  if (o.cls_cols) {
    cls = c0 / o.cls_cols;
    col = c0 - cls * o.cls_cols;
  }
  const int py = cls / o.xs, px = cls - py * o.xs;
  const int hh = h * o.ys + py, ww = w * o.xs + px;
  ShLoc l;
  l.valid = hh < o.vh && ww < o.vw;
  l.row = b * o.ob + (hh % o.hp) * o.ohp + (hh / o.hp) * o.oh + (ww / o.wp) * o.ow;
  l.dcol = col + (ww % o.wp) * o.owc;
  l.col = col;
  return l;
}

// KS: FWD K steps per tile (the issue loop unrolls over it; 0 for WGRAD)
template <int BN, int KIND, int KS>
__global__ void __launch_bounds__(kShThreads, 1)
    shconv_kernel(const __grid_constant__ CUtensorMap m0, const __grid_constant__ CUtensorMap m1,
                  const __grid_constant__ CUtensorMap m2, const __grid_constant__ CUtensorMap m3,
                  const __grid_constant__ CUtensorMap mres, const __grid_constant__ ShArgs a, Epilogue ep,
                  int stages) {
  using C = ShCfg<BN, KIND>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tiles = smem;
  uint8_t* b_res = smem + stages * a.stage_bytes;                    // FWD: kt boxes of BN x 64
  const int res_bytes = KIND == kShFwd ? a.kt * BN * 128 : 0;
  uint8_t* staging = b_res + res_bytes;                               // FWD: one output block per epilogue warp
  const int stg_total = KIND == kShFwd ? kShEpiWarps * a.stg_bytes : 0;
  uint64_t* bars = reinterpret_cast<uint64_t*>(staging + stg_total);  // [stages] full, [stages] empty
  uint64_t* acc_full = bars + 2 * kShMaxStages;
  uint64_t* acc_empty = acc_full + C::kAcc;
  uint64_t* bres_full = acc_empty + C::kAcc;
  uint64_t* drain = bres_full + 1;                                    // the MMA thread's final commit
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* bias_s = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(drain + 2) + 15) & ~uintptr_t(15));  // FWD bias

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // WGRAD with the bias gradient: the epilogue warps read every stage too
  const bool bsum = KIND == kShWgrad && a.bias_rows > 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(smem_u32(&bars[s]), 1);
      mbar_init(smem_u32(&bars[kShMaxStages + s]), bsum ? 1 + kShEpiWarps : 1);
    }
    for (int b = 0; b < C::kAcc; ++b) {
      mbar_init(smem_u32(&acc_full[b]), 1);
      mbar_init(smem_u32(&acc_empty[b]), C::kEpiPerTile);
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
  pdl_wait();          // the previous kernel's outputs (this kernel's inputs) are visible from here on
  pdl_trigger();
  if (KIND == kShFwd && ep.bias && threadIdx.x >= 64 && threadIdx.x < 64 + 128) {
    const int i = threadIdx.x - 64;
    bias_s[i] = i < a.N / a.nblk ? ep.bias[i] : 0.0f;
  }
  __syncthreads();
  // work units of this CTA: FWD tiles; WGRAD (n tile, k split) pairs
  const int nunits = KIND == kShFwd ? a.mt : a.nt * a.splits;
  auto unit_range = [&](int t, int* n0, int* k0, int* nk) {       // WGRAD: n tile and load-unit range of unit t
    const int nb = t % a.nt, sp = t / a.nt;
    *n0 = nb * BN;
    *k0 = sp * a.per;
    *nk = min(a.kt, *k0 + a.per) - *k0;
  };

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer
      if (KIND == kShFwd && static_cast<int>(blockIdx.x) < nunits) {
        const uint32_t rb = smem_u32(bres_full);
        mbar_expect_tx(rb, a.kt * BN * 128);
        for (int kb = 0; kb < a.kt; ++kb) tma_load_2d(smem_u32(b_res + kb * BN * 128), &mres, kb * 64, 0, rb);
      }
      int it = 0;
      bool stop = false;
      for (int t = blockIdx.x; t < nunits && !stop && !*abort; t += gridDim.x) {
        int first = t, count = 1;
        if (KIND == kShWgrad) {
          int n0;
          unit_range(t, &n0, &first, &count);
        }
        for (int i = 0; i < count; ++i, ++it) {
          const int s = it % stages;
          if (it >= stages && !mbar_wait(smem_u32(&bars[kShMaxStages + s]), ((it / stages) & 1) ^ 1, ep.err, 1, abort)) {
            stop = true;
            break;
          }
          if (ep.trace && blockIdx.x == 0 && it < kTraceN) ep.trace[it] = globaltimer();
          const uint32_t full = smem_u32(&bars[s]);
          mbar_expect_tx(full, a.unit_bytes);
          const uint32_t dst = smem_u32(tiles + s * a.stage_bytes);
          const int u = first + i;
          for (int g = 0; g < a.nseg_a + a.nseg_b; ++g) {
            const ShSeg& sg = a.seg[g];
            const int row = seg_row(sg, u);
            if (sg.gw)
              tma_load_3d(dst + sg.soff, pick(g, &m0, &m1, &m2, &m3), 0, 0, row / sg.gw, full);
            else
              tma_load_2d(dst + sg.soff, pick(g, &m0, &m1, &m2, &m3), 0, row, full);
          }
        }
      }
      if (*abort) {
        // copies may still be landing in stages nobody consumes: wait for
        // them (bounded) before the CTA's shared memory goes away
        for (int j = it > stages ? it - stages : 0; j < it; ++j)
          mbar_wait_bounded(smem_u32(&bars[j % stages]), (j / stages) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer (descriptor start addresses advance by (bytes >> 4) in the low field)
      bool ok = true;
      if (KIND == kShFwd && static_cast<int>(blockIdx.x) < nunits) {
        ok = mbar_wait(smem_u32(bres_full), 0, ep.err, 5, abort);
        fence_after();
      }
      const uint64_t db_res = smem_desc(smem_u32(b_res), 16, 1024);
      // FWD: every K step's A descriptor offset (descriptor units), loaded once
      uint32_t aoffs[KS > 0 ? KS : 1];
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) aoffs[ks] = static_cast<uint32_t>((ep.dbg & 16) ? (ks & 3) * 32 : a.a_koff[ks]) >> 4;
      int it = 0, tc = 0;
      for (int t = blockIdx.x; ok && t < nunits && !*abort; t += gridDim.x, ++tc) {
        const int buf = tc % C::kAcc, use = tc / C::kAcc;
        if (use > 0 && !mbar_wait(smem_u32(&acc_empty[buf]), (use & 1) ^ 1, ep.err, 4, abort)) break;
        fence_after();
        const uint32_t dtm = tmem + buf * BN;
        if (KIND == kShFwd) {
          const int s = it % stages;
          if (!mbar_wait(smem_u32(&bars[s]), (it / stages) & 1, ep.err, 2, abort)) break;
          fence_after();
          if (ep.trace && blockIdx.x == 0 && it < kTraceN) ep.trace[kTraceN + it] = globaltimer();
          const uint32_t stage = smem_u32(tiles + s * a.stage_bytes);
          const uint64_t da0 = smem_desc(stage, a.a_lbo, a.a_sbo, a.a_layout);
          constexpr uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) |
                                     (static_cast<uint32_t>(BM >> 4) << 24);
          if (!(ep.dbg & 2)) {
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
              constexpr uint32_t kBlk = BN * 128 / 16;     // one resident 64-wide K block, descriptor units
              mma_bf16(dtm, da0 + aoffs[ks], db_res + (ks >> 2) * kBlk + (ks & 3) * 2, idesc, ks > 0 ? 1u : 0u);
            }
          }
          mma_commit(smem_u32(&bars[kShMaxStages + s]));
          if (ep.trace && blockIdx.x == 0 && it < kTraceN) ep.trace[2 * kTraceN + it] = globaltimer();
          ++it;
        } else {
          int n0, k0, nk;
          unit_range(t, &n0, &k0, &nk);
          // MMA groups per N tile: one (BN 64) or two (BN 256, 384), fixed by the instantiation
          constexpr int NG = BN == 64 ? 1 : 2;
          const int g0 = n0 / a.subw;
          const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 15) | (1u << 16) |
                                 (static_cast<uint32_t>(a.subw >> 3) << 17) | (static_cast<uint32_t>(BM >> 4) << 24);
          const uint32_t ka = a.a_krow, kb = a.b_krow;     // 16 k-rows = (16 * krow) bytes = krow descriptor units
          const uint32_t all = (1u << a.ksteps) - 1u;
          bool good = true;
          for (int i = 0; i < nk; ++i, ++it) {
            const int s = it % stages;
            // K steps worth issuing: the grid rows of kmask (the unit's first step always issues)
            uint32_t issue = all;
            if (a.kgrid) {
              int h = (seg_row(a.seg[0], k0 + i) >> 4) % a.kgrid;
              if (h < 0) h += a.kgrid;
              issue = 0;
              for (int ks = 0; ks < a.ksteps; ++ks) {
                issue |= ((static_cast<uint32_t>(a.kmask) >> h) & 1u) << ks;
                h = h + 1 == a.kgrid ? 0 : h + 1;
              }
              if (i == 0) issue |= 1u;
            }
            if (!mbar_wait(smem_u32(&bars[s]), (it / stages) & 1, ep.err, 2, abort)) { good = false; break; }
            fence_after();
            if (ep.trace && blockIdx.x == 0 && it < kTraceN) ep.trace[kTraceN + it] = globaltimer();
            const uint32_t stage = smem_u32(tiles + s * a.stage_bytes);
            const uint64_t da0 = smem_desc(stage + a.a_off, a.a_lbo, a.a_sbo, a.a_layout);
            uint64_t db0[NG];
#pragma unroll
            for (int j = 0; j < NG; ++j) db0[j] = smem_desc(stage + a.b_noff[g0 + j], a.b_lbo, a.b_sbo, a.b_layout);
            if (!(ep.dbg & 2)) {
              uint32_t acc = i > 0 ? 1u : 0u;
#pragma unroll 4
              for (int ks = 0; ks < a.ksteps; ++ks) {
                if (!((issue >> ks) & 1u)) continue;
#pragma unroll
                for (int j = 0; j < NG; ++j) mma_bf16(dtm + j * a.subw, da0 + ks * ka, db0[j] + ks * kb, idesc, acc);
                acc = 1u;
              }
            }
            mma_commit(smem_u32(&bars[kShMaxStages + s]));
            if (ep.trace && blockIdx.x == 0 && it < kTraceN) ep.trace[2 * kTraceN + it] = globaltimer();
          }
          if (!good) break;
        }
        mma_commit(smem_u32(&acc_full[buf]));
      }
      // every MMA issued by this thread has completed before the tensor memory is freed
      mma_commit(smem_u32(drain));
      mbar_wait_bounded(smem_u32(drain), 0);
    }
  } else if (KIND == kShFwd) {
    // ---- epilogue warps 2..9, FWD: the halves take alternate tiles; each
    // warp writes the output rows of its TMEM lane quadrant into its own
    // shared-memory block (one contiguous range of the destination: the
    // caller's maps guarantee it) and copies the block out with coalesced
    // 16-byte stores; for the input gradients the saved activation of the
    // same block is fetched into it first (cp.async, issued before the
    // accumulator is waited for) and the result overwrites it in place
    const int quad = warp & 3, half = (warp - 2) >> 2, ew = warp - 2;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    uint8_t* stg = staging + ew * a.stg_bytes;
    const uint32_t stg_s = smem_u32(stg);
    const bool grad = ep.act == kReluGrad;
    const int nb = a.N / a.nblk;                 // output columns (<= 128: at most 4 chunks of 32)
    const ShOut& o = a.om;
    const int64_t rbytes = ep.ldc * 2;
    // a tile is one image (gw * gh == BM), so a lane's grid position and the
    // destination of each of its chunks differ between tiles only by the
    // image's row offset: locate them once
    const int r = quad * 32 + lane, h = r / o.gw, w = r - (r / o.gw) * o.gw;
    int64_t roff[4];
    int dcol[4], ccol[4];
    bool cvalid[4], cwrite[4];
    long long lo0 = LLONG_MAX, hi0 = -1;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const ShLoc l = sh_locate(o, 0, h, w, c * 32);
      roff[c] = l.row;
      dcol[c] = l.dcol;
      ccol[c] = l.col;
      cvalid[c] = l.valid;
      cwrite[c] = c * 32 < nb && (l.valid || a.zero_fill);
      if (cwrite[c]) {
        lo0 = min(lo0, static_cast<long long>(l.row));
        hi0 = max(hi0, static_cast<long long>(l.row));
      }
    }
#pragma unroll
    for (int sh = 16; sh > 0; sh >>= 1) {
      lo0 = min(lo0, __shfl_xor_sync(0xffffffffu, lo0, sh));
      hi0 = max(hi0, __shfl_xor_sync(0xffffffffu, hi0, sh));
    }
    const int chunks = hi0 >= lo0 ? static_cast<int>((hi0 - lo0 + 1) * rbytes / 16) : 0;
    const bool fits = chunks * 16 <= a.stg_bytes;
    if (!fits && lane == 0 && blockIdx.x == 0) atomicCAS(ep.err, 0, 6);
    int tc = 0;
    for (int t = blockIdx.x; t < nunits; t += gridDim.x, ++tc) {
      if ((tc & 1) != half) continue;
      const int buf = tc % C::kAcc, use = tc / C::kAcc;
      const bool in_rows = t * BM + r < a.M;
      const long long lo = lo0 + static_cast<long long>(t) * o.ob;
      const bool active = chunks > 0 && fits && !(ep.dbg & 1);
      if (grad && active) {
        const uint8_t* src = reinterpret_cast<const uint8_t*>(ep.aux + lo * ep.ld_aux);
#pragma unroll 4
        for (int i = lane; i < chunks; i += 32) cp_async16(stg_s + stg_chunk(i) * 16, src + i * 16);
        asm volatile("cp.async.commit_group;" ::: "memory");
      }
      const bool xt = ep.trace && (ep.dbg & 64) && blockIdx.x == 0 && warp == 2 && lane == 0 && tc < kTraceN;
      if (xt) ep.trace[5 * kTraceN + tc] = globaltimer();
      const bool got = mbar_wait(smem_u32(&acc_full[buf]), use & 1, ep.err, 3, abort, true);
      if (grad && active) {
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        __syncwarp();
      }
      if (!got) break;
      fence_after();
      if (ep.trace && blockIdx.x == 0 && warp == 2 && lane == 0 && tc < kTraceN) ep.trace[3 * kTraceN + tc] = globaltimer();
      if (!(ep.dbg & 32)) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if (c * 32 >= nb) break;
          const int c0 = c * 32;
          float v[32];
          tmem_ld32(lane_base + buf * BN + c0, v);
          if (xt && c == 0) ep.trace[6 * kTraceN + tc] = globaltimer();
          // row stacking: block j of row q + bd[j] belongs to this row
#pragma unroll 1
          for (int j = 1; j < a.nblk; ++j) {
            float u[32];
            tmem_ld32(lane_base + buf * BN + j * nb + c0, u);
            const int d = a.bd[j];
            const bool inside = lane + d < 32;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float x = __shfl_down_sync(0xffffffffu, u[i], d);
              v[i] += inside ? x : 0.0f;
            }
          }
          if (active && in_rows && cwrite[c]) {
            uint4* slots = reinterpret_cast<uint4*>(stg);
            const int i0 = static_cast<int>(((roff[c] - lo0) * rbytes + dcol[c] * 2) >> 4);
            if (!cvalid[c]) {
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = 0.0f;
            } else {
              if (ep.bias) {
                const float4* b4 = reinterpret_cast<const float4*>(bias_s + ccol[c]);   // per output channel
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                  const float4 bb = b4[i];
                  v[4 * i] += bb.x; v[4 * i + 1] += bb.y; v[4 * i + 2] += bb.z; v[4 * i + 3] += bb.w;
                }
              }
              if (ep.act == kRelu) {
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = fmaxf(v[i], 0.0f);
              } else if (grad) {
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  const uint4 wv = slots[stg_chunk(i0 + q)];
                  const uint32_t ww4[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                  for (int k = 0; k < 4; ++k) {
                    if (!(__uint_as_float(ww4[k] << 16) > 0.0f)) v[8 * q + 2 * k] = 0.0f;
                    if (!(__uint_as_float(ww4[k] & 0xFFFF0000u) > 0.0f)) v[8 * q + 2 * k + 1] = 0.0f;
                  }
                }
              }
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint32_t pk[4];
#pragma unroll
              for (int k = 0; k < 4; ++k)
                pk[k] = surfk::pack_bf16x2(v[8 * q + 2 * k], v[8 * q + 2 * k + 1]);
              slots[stg_chunk(i0 + q)] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            }
          }
        }
        __syncwarp();
        if (xt) ep.trace[7 * kTraceN + tc] = globaltimer();
        if (active) {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(ep.c) + lo * rbytes);
          const uint4* src = reinterpret_cast<const uint4*>(stg);
#pragma unroll 4
          for (int i = lane; i < chunks; i += 32) dst[i] = src[stg_chunk(i)];
        }
        __syncwarp();
      }
      fence_before();
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&acc_empty[buf])) : "memory");
      if (ep.trace && blockIdx.x == 0 && warp == 2 && lane == 0 && tc < kTraceN) ep.trace[4 * kTraceN + tc] = globaltimer();
    }
  } else {
    // ---- epilogue warps 2..9, WGRAD: the halves split the unit's columns;
    // while the MMAs run they sum the output gradient's rows of every stage
    // (the bias gradient; lane l owns columns 2l, 2l + 1, warp w rows w + 8i)
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2, ew = warp - 2;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    float bs0 = 0.0f, bs1 = 0.0f;
    int tc = 0, it = 0;
    bool dead = false;
    for (int t = blockIdx.x; t < nunits; t += gridDim.x, ++tc) {
      const int buf = tc % C::kAcc, use = tc / C::kAcc;
      const int c_first = 32 * half;
      if (bsum) {
        int n0u, k0u, nku;
        unit_range(t, &n0u, &k0u, &nku);
        for (int i = 0; i < nku; ++i, ++it) {
          const int s = it % stages;
          if (!mbar_wait(smem_u32(&bars[s]), (it / stages) & 1, ep.err, 8, abort)) {
            dead = true;
            break;
          }
          if (n0u == 0) {
            const uint8_t* box = tiles + s * a.stage_bytes + a.seg[0].soff;
            const int cb = lane * 4;                       // byte of the column pair in the row
#pragma unroll 4
            for (int r = ew; r < a.bias_rows; r += kShEpiWarps) {
              const uint32_t x =
                  *reinterpret_cast<const uint32_t*>(box + r * 128 + (((cb >> 4) ^ (r & 7)) << 4) + (cb & 15));
              bs0 += __uint_as_float(x << 16);
              bs1 += __uint_as_float(x & 0xFFFF0000u);
            }
          }
          __syncwarp();
          if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&bars[kShMaxStages + s])) : "memory");
        }
        if (dead) break;
      }
      if (!mbar_wait(smem_u32(&acc_full[buf]), use & 1, ep.err, 3, abort, true)) break;
      fence_after();
      if (ep.trace && blockIdx.x == 0 && warp == 2 && lane == 0 && tc < kTraceN) ep.trace[3 * kTraceN + tc] = globaltimer();
      int n0, k0, nk;
      unit_range(t, &n0, &k0, &nk);
      const int rowoff = a.erow[quad];
#pragma unroll 1
      for (int c0 = c_first; c0 < BN && !(ep.dbg & 32); c0 += 64) {
        if (n0 + c0 >= a.N) break;
        float v[32];
        tmem_ld32(lane_base + buf * BN + c0, v);
        if (!(ep.dbg & 1)) {
#pragma unroll
          for (int hb = 0; hb < 2; ++hb) {
            const int n = n0 + c0 + 16 * hb;
            const int col = n < a.N ? a.ecol[quad][n >> 4] : -1;
            if (col >= 0) {
              float* dst = static_cast<float*>(ep.c) + static_cast<int64_t>(lane + rowoff) * ep.ldc + col;
#pragma unroll
              for (int i = 0; i < 16; i += 4)
                asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst + i), "f"(v[16 * hb + i]),
                             "f"(v[16 * hb + i + 1]), "f"(v[16 * hb + i + 2]), "f"(v[16 * hb + i + 3])
                             : "memory");
            }
          }
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&acc_empty[buf])) : "memory");
      if (ep.trace && blockIdx.x == 0 && warp == 2 && lane == 0 && tc < kTraceN) ep.trace[4 * kTraceN + tc] = globaltimer();
    }
    if (bsum && !(ep.dbg & 1)) {
      float* gb = static_cast<float*>(ep.ct);
      atomicAdd(gb + (2 * lane) % a.bias_mod, bs0);
      atomicAdd(gb + (2 * lane + 1) % a.bias_mod, bs1);
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::kTmemCols));
}

// weight rearrangement for the stacked B operands: out[i] = src[idx[i]] (0 where idx < 0)
__global__ void gather_weights_kernel(const uint16_t* __restrict__ src, const int* __restrict__ idx,
                                      uint16_t* __restrict__ out, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int k = idx[i];
    out[i] = k >= 0 ? src[k] : static_cast<uint16_t>(0);
  }
}

// ---- host side -------------------------------------------------------------------
struct ShMap {               // a bf16 view of `rows` grid rows of `inner` elements (dense rows)
  const void* base;
  int64_t rows;
  int inner;                 // 16, 32 or 64 elements (32, 64 or 128 bytes)
  int gw;                    // 0: 2-D; else rows come in groups of gw ...
  int64_t gstride;           // ... gstride bytes apart (a plane of every other grid row)
};

struct ShDesc {
  ShArgs a;
  ShMap maps[4];             // map g serves box g (A boxes first, then B boxes)
  ShMap res;                 // FWD: weights [N rows][K], read as boxes of 64 x BN
  int64_t res_ld;            // elements between weight rows
  int bn;
};

CUtensorMapSwizzle swz_for(int bytes) {
  return bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B : bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
}

// 3-D bf16 map: (inner, gw, rows / gw) with row stride inner and group stride gstride bytes
bool make_map3(CUtensorMap* m, const ShMap& s, int box_rows) {
  auto fn = encode_fn();
  if (!fn || s.gw < 1 || s.rows % s.gw || box_rows % s.gw || (s.gstride & 15)) return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(s.inner), static_cast<cuuint64_t>(s.gw),
                        static_cast<cuuint64_t>(s.rows / s.gw)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(s.inner) * 2, static_cast<cuuint64_t>(s.gstride)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(s.inner), static_cast<cuuint32_t>(s.gw),
                       static_cast<cuuint32_t>(box_rows / s.gw)};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(s.base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swz_for(s.inner * 2), CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int KIND, int KS>
int sh_launch(const ShDesc& d, const Epilogue& ep, cudaStream_t s) {
  const ShArgs& a = d.a;
  CUtensorMap mp[4], mres;
  std::memset(mp, 0, sizeof mp);
  std::memset(&mres, 0, sizeof mres);
  for (int g = 0; g < a.nseg_a + a.nseg_b; ++g) {
    const ShMap& m = d.maps[g];
    const ShSeg& sg = a.seg[g];
    if (!m.base || (reinterpret_cast<uintptr_t>(m.base) & 15) || m.inner * 2 != sg.row_bytes || sg.rows < 1 ||
        (sg.soff & 1023) || sg.gw != m.gw)
      return static_cast<int>(cudaErrorInvalidValue);
    if (m.gw) {
      // 3-D box: whole groups, every unit's first row a group boundary
      if (sg.rows / m.gw > 256 || m.gw > 256 || sg.mul_hi % m.gw || sg.mul_lo % m.gw || sg.add % m.gw ||
          !make_map3(&mp[g], m, sg.rows))
        return static_cast<int>(cudaErrorInvalidValue);
    } else {
      if (sg.rows > 256 ||
          !make_map(&mp[g], m.base, m.inner, m.rows, m.inner, m.inner, sg.rows, false, swz_for(m.inner * 2)))
        return static_cast<int>(cudaErrorInvalidValue);
    }
  }
  if (KIND == kShFwd) {
    if (!d.res.base || !make_map(&mres, d.res.base, d.res.inner, d.res.rows, d.res_ld, 64, BN))
      return static_cast<int>(cudaErrorInvalidValue);
  } else {
    mres = mp[0];
  }
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  const int res_bytes = KIND == kShFwd ? a.kt * BN * 128 : 0;
  const int stg_total = KIND == kShFwd ? kShEpiWarps * a.stg_bytes : 0;
  const int budget = 232448 - 1024 - 1024 - res_bytes - stg_total;
  int stages = budget / a.stage_bytes;
  if (stages > kShMaxStages) stages = kShMaxStages;
  if (stages < 2) return static_cast<int>(cudaErrorInvalidValue);
  const size_t smem = 1024 + static_cast<size_t>(stages) * a.stage_bytes + res_bytes + stg_total + 1024;
  auto kern = shconv_kernel<BN, KIND, KS>;
  // the largest dynamic size any call of this instantiation asks for, set
  // once per device: several layers share an instantiation with different
  // stage counts, and a graph node captured with a larger size must not meet
  // an attribute lowered by a later call
  const cudaError_t attr = smem_limit_once<shconv_kernel<BN, KIND, KS>>(232448);
  if (attr != cudaSuccess) return static_cast<int>(attr);
  const int units = KIND == kShFwd ? a.mt : a.nt * a.splits;
  const int grid = units < sms ? units : sms;
  launch_pdl(kern, dim3(grid), dim3(kShThreads), smem, s, mp[0], mp[1], mp[2], mp[3], mres, a, ep, stages);
  SURF_RETURN_LAUNCH();
}

}  // namespace

// One convolution GEMM over shifted row views (see the file comment). The
// caller (ops/conv_shift.py) builds the boxes, descriptor offsets, stacking
// and output maps of the layer; this entry point validates the ranges it
// can (every operand inside its stage, every table index in range), encodes
// the tensor maps and launches.
SURF_EXPORT int surf_shconv(const ShDesc* d, const Epilogue* ep, void* stream) {
  const ShArgs& a = d->a;
  if (a.kind != kShFwd && a.kind != kShWgrad) return static_cast<int>(cudaErrorInvalidValue);
  if (a.nseg_a < 1 || a.nseg_a + a.nseg_b > 4 || a.nseg_b < 0 || a.stage_bytes < 1024 || (a.stage_bytes & 1023))
    return static_cast<int>(cudaErrorInvalidValue);
  if (a.M <= 0 || a.N <= 0 || a.kt <= 0) return 0;
  int landed = 0;
  for (int g = 0; g < a.nseg_a + a.nseg_b; ++g) {
    if (a.seg[g].udiv < 1 || a.seg[g].soff + a.seg[g].rows * a.seg[g].row_bytes > a.stage_bytes)
      return static_cast<int>(cudaErrorInvalidValue);
    landed += a.seg[g].rows * a.seg[g].row_bytes;
  }
  if (landed != a.unit_bytes) return static_cast<int>(cudaErrorInvalidValue);
  if (a.kind == kShFwd) {
    if (a.N > d->bn || a.ksteps < 1 || a.ksteps > a.kt * 4 || a.ksteps <= (a.kt - 1) * 4 ||
        a.ksteps > kShMaxKSteps || a.mt * BM < a.M || !ep->c || ep->c_dtype != 1 || (ep->act == kReluGrad && !ep->aux) ||
        a.om.gw < 1 || a.om.gh < 1 || a.om.hp < 1 || a.om.wp < 1 || a.om.xs < 1 || a.om.ys < 1 ||
        (a.om.cls_cols & 31) || a.nblk < 1 || a.nblk > 4 || a.N % a.nblk || (a.N / a.nblk) % 32 ||
        a.stg_bytes < 128 || (a.stg_bytes & 127) || (reinterpret_cast<uintptr_t>(ep->c) & 15) ||
        a.om.gw * a.om.gh != BM || a.N / a.nblk > 128 ||
        (ep->act == kReluGrad && (ep->ld_aux != ep->ldc || (reinterpret_cast<uintptr_t>(ep->aux) & 15))))
      return static_cast<int>(cudaErrorInvalidValue);
    for (int j = 0; j < a.nblk; ++j)
      if (a.bd[j] < 0 || a.bd[j] > 31) return static_cast<int>(cudaErrorInvalidValue);
    const int rb = a.seg[0].row_bytes;               // every A operand reads 128 rows from its offset
    for (int k = 0; k < a.ksteps; ++k)
      if (a.a_koff[k] < 0 || a.a_koff[k] - a.a_koff[k] % rb + BM * rb > a.stage_bytes)
        return static_cast<int>(cudaErrorInvalidValue);
  } else {
    if (a.subw < 16 || a.subw > 256 || (a.subw & 15) || d->bn % a.subw || a.splits < 1 || a.per < 1 ||
        a.nt * d->bn < a.N || a.N > 16 * kShMaxNb16 || (a.N + a.subw - 1) / a.subw > kShMaxSub || !ep->c ||
        ep->c_mode != kAtomic || a.ksteps < 1 || (reinterpret_cast<uintptr_t>(ep->c) & 15) || (ep->ldc & 3) ||
        (a.bias_rows > 0 && (!ep->ct || a.seg[0].row_bytes != 128 || a.bias_rows > a.seg[0].rows ||
                             a.bias_mod < 1 || a.bias_mod > 64)) ||
        (a.kgrid && (a.kgrid > 32 || a.kgrid < 1 || a.seg[0].udiv != 1 || (a.seg[0].mul_hi & 15) || (a.seg[0].add & 15))) ||
        a.ksteps > 32 || d->bn / a.subw != (d->bn == 64 ? 1 : 2) || a.nt != 1)
      return static_cast<int>(cudaErrorInvalidValue);
    // every MMA operand (the K steps' 16-row slices, both MN blocks of A and
    // every N block of a group) lies inside one stage
    const int a_end = a.a_off + a.a_lbo + (a.ksteps * 16) * a.a_krow;
    if (a.a_off < 0 || a.a_lbo < 0 || a_end > a.stage_bytes) return static_cast<int>(cudaErrorInvalidValue);
    const int blocks = a.subw / (a.b_krow / 2);      // MN blocks of one MMA group, b_lbo apart
    for (int g = 0; g < (a.N + a.subw - 1) / a.subw; ++g)
      if (a.b_noff[g] < 0 || a.b_noff[g] + (blocks - 1) * a.b_lbo + a.ksteps * 16 * a.b_krow > a.stage_bytes)
        return static_cast<int>(cudaErrorInvalidValue);
  }
  auto s = static_cast<cudaStream_t>(stream);
  if (a.kind == kShFwd) {
    // the trunk's forward-kind shapes: (N, K steps)
    const int key = d->bn * 100 + a.ksteps;
    switch (key) {
      case 128 * 100 + 10: return sh_launch<128, kShFwd, 10>(*d, *ep, s);   // conv1 forward
      case 128 * 100 + 16: return sh_launch<128, kShFwd, 16>(*d, *ep, s);   // conv2 forward
      case 192 * 100 + 12: return sh_launch<192, kShFwd, 12>(*d, *ep, s);   // conv3 forward, input gradient
      case 256 * 100 + 8: return sh_launch<256, kShFwd, 8>(*d, *ep, s);     // conv2 input gradient
      default: return static_cast<int>(cudaErrorInvalidValue);
    }
  }
  switch (d->bn) {
    case 64: return sh_launch<64, kShWgrad, 0>(*d, *ep, s);
    case 256: return sh_launch<256, kShWgrad, 0>(*d, *ep, s);
    case 384: return sh_launch<384, kShWgrad, 0>(*d, *ep, s);
    default: return static_cast<int>(cudaErrorInvalidValue);
  }
}

// out[i] = src[idx[i]] (0 where idx[i] < 0): the stacked weight operands,
// rebuilt from the bf16 parameters after every optimizer step
SURF_EXPORT int surf_shconv_weights(const void* src, const int* idx, void* out, int64_t n, void* stream) {
  if (n <= 0) return 0;
  if (!src || !idx || !out) return static_cast<int>(cudaErrorInvalidValue);
  const int64_t blocks = (n + 255) / 256;
  gather_weights_kernel<<<static_cast<int>(blocks < 1184 ? blocks : 1184), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(src), idx, static_cast<uint16_t*>(out), n);
  SURF_RETURN_LAUNCH();
}

SURF_EXPORT int surf_shconv_sizes(int* out) {
  out[0] = static_cast<int>(sizeof(ShDesc));
  out[1] = static_cast<int>(sizeof(ShArgs));
  out[2] = static_cast<int>(sizeof(ShSeg));
  out[3] = static_cast<int>(sizeof(ShOut));
  out[4] = static_cast<int>(sizeof(ShMap));
  return 0;
}
