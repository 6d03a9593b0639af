// tc_sm100.cuh — shared pieces of the tcgen05 GEMM kernels (sm_100a): the
// epilogue description, PTX wrappers (mbarriers, TMA, UMMA descriptors,
// tcgen05.mma / commit / ld), the fused bias / activation epilogue of a
// 32-column accumulator chunk and its register-path stores, and the host-side
// 2-D tensor-map encoder. Included by gemm_tc.cu (the general GEMM and
// implicit convolutions over 4-D maps) and conv_shift.cu (convolutions on
// row-shifted views of flattened activation grids); everything sits in an
// anonymous namespace, so each translation unit has its own copy.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <utility>

#include "surf_cuda.cuh"

namespace {

constexpr int BM = 128, BK = 64;
constexpr uint64_t kWaitNs = 2000000000ull;    // 2 s bound per barrier wait

enum Act : int { kNone = 0, kRelu = 1, kTanh = 2, kReluGrad = 3, kTanhGrad = 4 };
enum CMode : int { kStore = 0, kAtomic = 1 };

struct Epilogue {
  void* c;            // [M, N] output (or null)
  int64_t ldc;
  int c_dtype;        // 0 fp32, 1 bf16
  int c_mode;         // 0 store, 1 fp32 atomic add
  void* ct;           // optional transposed output [N, M]
  int64_t ldct;
  int ct_dtype;
  const float* bias;  // [N] or null
  int act;            // activation for columns < act_split
  int act2;           // activation for columns >= act_split
  int act_split;
  const uint16_t* aux;   // bf16 [M, N] saved activation for the derivative modes
  int64_t ld_aux;
  int* err;           // device error flag (0 = ok)
  int dbg;            // diagnostics (timing studies only): bit 0 skip epilogue stores, bit 1 skip MMAs,
                      // bit 2 stream a resident-able B per k-block, bit 3 no saved-activation prefetch
  // diagnostics: CTA 0 records %globaltimer stamps of its first kTraceN
  // k-blocks / tiles here (null: off): [0,N) producer issue, [N,2N) TMA
  // landed (seen by the MMA warp), [2N,3N) MMAs committed, [3N,4N) tile
  // accumulator ready (epilogue warp 2), [4N,5N) tile epilogue done
  unsigned long long* trace;
  // column remap of the stored output (0: off): column n goes to
  // (n / cmap_in) * cmap_out + n % cmap_in -- e.g. a dense h x w x c row
  // written onto a wider zero-padded grid; the saved activation and the bias
  // keep the dense column
  int cmap_in, cmap_out;
};
constexpr int kTraceN = 256;

// ---- PTX wrappers --------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait that may suspend the thread up to `ns` nanoseconds (it resumes as
// soon as the phase completes): waiting warps stop competing for issue slots
__device__ __forceinline__ bool mbar_try_sleep(uint32_t bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}
// Bounded wait; returns false (and records `code`) on timeout or when another
// role already gave up (*abort set).
// `nap`: waits off the critical path (epilogue warps waiting for an
// accumulator) may suspend between polls
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err, int code, volatile int* abort,
                                          bool nap = false) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (nap ? mbar_try_sleep(bar, parity, 20000u) : mbar_try(bar, parity)) return true;
    if ((i & 255) == 0) {
      if (*abort) return false;
      if (globaltimer() - t0 > kWaitNs) {
        if (err) atomicCAS(err, 0, code);
        *abort = 1;
        return false;
      }
    }
  }
}

// wait on an mbarrier phase for at most the usual bound, whatever the abort
// flag says (the abort paths' drains of work still in flight)
__device__ __forceinline__ void mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try(bar, parity))
    if (globaltimer() - t0 > kWaitNs) return;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int c, int w, int h, int b,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(c), "r"(w), "r"(h), "r"(b), "r"(bar)
      : "memory");
}

// Shared-memory matrix descriptor (sm100 UMMA): start, LBO, SBO (>> 4),
// descriptor version 1, layout type (2: 128-byte, 4: 64-byte, 6: 32-byte swizzle).
constexpr uint32_t kSw128 = 2, kSw64 = 4, kSw32 = 6;
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo, uint32_t layout = kSw128) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32;
  d |= 1ull << 46;
  d |= static_cast<uint64_t>(layout & 7) << 61;
  return d;
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accum), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr + 16));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(src)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// tanh through the hardware's approximate tanh (one MUFU instruction,
// relative error about 2^-11: below a bf16 output's half ulp of 2^-9 for
// most values, at the level of the exp-based form it replaces for fp32
// outputs). The exact-division form took ~15 instructions per element and
// showed in the epilogue of the 32768-row tanh layers.
__device__ __forceinline__ float tanh_fast(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Bias + activation (or activation derivative) for a 32-column chunk of one
// row. The activation is chosen once per chunk (act_split is a multiple of
// 32), bias and the saved activation are loaded with vector loads, and each
// activation has its own tight loop.
__device__ __forceinline__ void process_chunk32(const Epilogue& ep, float* v, int64_t row, bool row_ok, int col0,
                                                int N, const uint4* pre = nullptr) {
  const bool full = col0 + 32 <= N;
  if (ep.bias) {
    if (full) {
      const float4* b4 = reinterpret_cast<const float4*>(ep.bias + col0);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 b = __ldg(b4 + i);
        v[4 * i] += b.x; v[4 * i + 1] += b.y; v[4 * i + 2] += b.z; v[4 * i + 3] += b.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (col0 + i < N) v[i] += __ldg(ep.bias + col0 + i);
    }
  }
  const int act = col0 < ep.act_split ? ep.act : ep.act2;
  if (act == kNone) return;
  if (act == kRelu) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = fmaxf(v[i], 0.0f);
    return;
  }
  if (act == kTanh) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = tanh_fast(v[i]);
    return;
  }
  // derivative modes: aux = saved bf16 activation of this row
  float a[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) a[i] = 0.0f;
  if (pre) {
    // loaded ahead by load_aux32 (a full, aligned chunk of a valid row)
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t ww[4] = {pre[q].x, pre[q].y, pre[q].z, pre[q].w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        a[8 * q + 2 * k] = __uint_as_float(ww[k] << 16);
        a[8 * q + 2 * k + 1] = __uint_as_float(ww[k] & 0xFFFF0000u);
      }
    }
  } else if (row_ok) {
    const uint16_t* src = ep.aux + row * ep.ld_aux + col0;
    if (full && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 w = *reinterpret_cast<const uint4*>(src + 8 * q);
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          a[8 * q + 2 * k] = __uint_as_float(ww[k] << 16);
          a[8 * q + 2 * k + 1] = __uint_as_float(ww[k] & 0xFFFF0000u);
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (col0 + i < N) a[i] = surfk::bf16_to_f32(src[i]);
    }
  }
  if (act == kReluGrad) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = a[i] > 0.0f ? v[i] : 0.0f;
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = v[i] * (1.0f - a[i] * a[i]);
  }
}

// Saved-activation row of a derivative-mode chunk, loaded ahead of its
// accumulator (4 x 16 bytes); false (nothing loaded) for other activations,
// invalid rows, partial or unaligned chunks, which process_chunk32 loads itself.
__device__ __forceinline__ bool load_aux32(const Epilogue& ep, int64_t row, bool row_ok, int col0, int N,
                                           uint4 (&w)[4]) {
  const int act = col0 < ep.act_split ? ep.act : ep.act2;
  if ((act != kReluGrad && act != kTanhGrad) || !row_ok || col0 + 32 > N) return false;
  const uint16_t* src = ep.aux + row * ep.ld_aux + col0;
  if (reinterpret_cast<uintptr_t>(src) & 15) return false;
#pragma unroll
  for (int q = 0; q < 4; ++q) w[q] = *reinterpret_cast<const uint4*>(src + 8 * q);
  return true;
}

// Register-path stores of a processed 32-column chunk (transposed output,
// fp32 atomics, or rows that TMA cannot address). Every loop over the chunk
// is fully unrolled with a column predicate: a loop with a run-time trip
// count would index v[] dynamically and put the whole accumulator chunk of
// every epilogue in local memory.
__device__ __forceinline__ void store_chunk32(const Epilogue& ep, const float* v, int64_t row, bool row_ok, int col0,
                                              int N) {
  if (!row_ok) return;
  const int ncol = min(32, N - col0);
  if (ep.ct) {
    // for a fixed column the warp's 32 lanes write 32 consecutive rows
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      if (i >= ncol) break;
      if (ep.ct_dtype == 1) static_cast<uint16_t*>(ep.ct)[(col0 + i) * ep.ldct + row] = surfk::f32_to_bf16(v[i]);
      else static_cast<float*>(ep.ct)[(col0 + i) * ep.ldct + row] = v[i];
    }
  }
  if (!ep.c) return;
  if (ep.cmap_in) col0 = (col0 / ep.cmap_in) * ep.cmap_out + col0 % ep.cmap_in;
  if (ep.c_mode == kAtomic) {
    float* dst = static_cast<float*>(ep.c) + row * ep.ldc + col0;
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i < ncol) atomicAdd(dst + i, v[i]);
  } else if (ep.c_dtype == 1) {
    uint16_t* dst = static_cast<uint16_t*>(ep.c) + row * ep.ldc + col0;
    if (ncol == 32 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
          w[k] = surfk::pack_bf16x2(v[8 * q + 2 * k], v[8 * q + 2 * k + 1]);
        reinterpret_cast<uint4*>(dst)[q] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < ncol) dst[i] = surfk::f32_to_bf16(v[i]);
    }
  } else {
    float* dst = static_cast<float*>(ep.c) + row * ep.ldc + col0;
    if (ncol == 32 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
      for (int i = 0; i < 8; ++i) reinterpret_cast<float4*>(dst)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < ncol) dst[i] = v[i];
    }
  }
}

// Programmatic dependent launch: a kernel launched with the programmatic
// stream-serialization attribute may start while the previous kernel of its
// stream drains; every thread calls pdl_wait() after its prologue (barrier
// set-up, tensor-memory allocation) and before it reads any input, which
// returns once the previous grid has completed and its writes are visible
// (a no-op for a normal launch). pdl_trigger() lets this kernel's own
// dependents start their prologues.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- host side ---------------------------------------------------------------
// Launch with programmatic stream serialization (SURF_NO_PDL=1: plain
// launch). Under a profiler's injection library (Nsight Compute sets
// CUDA_INJECTION64_PATH) the launches are plain too: a programmatic launch
// inside a captured graph failed to launch under ncu's kernel serialization.
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("SURF_NO_PDL");
    const char* inj = std::getenv("CUDA_INJECTION64_PATH");
    return !(e && e[0] == '1') && !(inj && inj[0]);
  }();
  return on;
}

// Raise kernel Kern's dynamic shared-memory limit to `bytes` once per device.
// The attribute belongs to the kernel in the current device's context, so a
// process that drives several GPUs sets it on each of them; after the first
// call on a device this is a device query and an atomic load.
template <auto Kern>
cudaError_t smem_limit_once(int bytes) {
  static std::atomic<uint64_t> done{0};    // bit d: set on device d (0..63)
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = dev >= 0 && dev < 64 ? uint64_t{1} << dev : 0;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  e = cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

template <typename... Exp, typename... Act>
cudaError_t launch_pdl(void (*kernel)(Exp...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Act&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Act>(args)...);
}
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D bf16 tensor map: `rows` x `inner` elements, row stride `ld` elements,
// box of box_inner x box_rows, 128-byte swizzle, zero fill out of bounds.
bool make_map(CUtensorMap* m, const void* base, int64_t inner, int64_t rows, int64_t ld, int box_inner, int box_rows,
              bool fp32 = false, CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto fn = encode_fn();
  if (!fn) return false;
  const int esize = fp32 ? 4 : 2;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * esize)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace
