// nn_ops.cu — the non-GEMM layers of the policy network (sm_100a).
//
//   * im2col: NHWC bf16 activations -> convolution patch rows (kh, kw, c order)
//     so that a convolution is one tensor-core GEMM;
//   * col2im_relu: the transposed scatter, written as a gather (no atomics,
//     8 channels per thread, only the stride-congruent taps visited), fused
//     with the ReLU derivative of the layer below;
//   * colsum: bias gradients (sum of dY over rows), fp32 accumulation;
//   * gather_rows: minibatch rows of the rollout buffers (any element size);
//   * frame_stack: the policy input of a decision from the frames of earlier
//     decisions (rollout, truncation bootstrap and minibatch gather);
//   * cast kernels between fp32 and bf16.
#include <cstdint>

#include "surf_cuda.cuh"

namespace {

struct ConvGeom {
  int B, H, W, C;      // input NHWC
  int KH, KW, S;       // kernel, stride (no padding)
  int OH, OW;
};

// One thread per (output pixel, kh, 8-element chunk of the kw*C run) of ONE
// image: blockIdx.y is the image, so all index math is 32-bit.
__global__ void im2col_kernel(const uint16_t* x, uint16_t* col, int64_t ldcol, ConvGeom g) {
  const int run = g.KW * g.C;                 // contiguous elements per kh
  const int chunks = (run + 7) / 8;
  const int per_image = g.OH * g.OW * g.KH * chunks;
  for (int b = blockIdx.y; b < g.B; b += gridDim.y) {
    const uint16_t* xb = x + static_cast<int64_t>(b) * g.H * g.W * g.C;
    uint16_t* cb = col + static_cast<int64_t>(b) * g.OH * g.OW * ldcol;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < per_image; i += gridDim.x * blockDim.x) {
      const int ch = i % chunks;
      const int r = i / chunks;
      const int kh = r % g.KH;
      const int pix = r / g.KH;               // oh * OW + ow
      const int ow = pix % g.OW, oh = pix / g.OW;
      const uint16_t* src = xb + ((oh * g.S + kh) * g.W + ow * g.S) * g.C;
      uint16_t* dst = cb + pix * ldcol + kh * run;
      const int e0 = ch * 8;
      const int n = min(8, run - e0);
      const uintptr_t al = reinterpret_cast<uintptr_t>(src + e0) | reinterpret_cast<uintptr_t>(dst + e0);
      if (n == 8 && (al & 15) == 0) {
        *reinterpret_cast<uint4*>(dst + e0) = __ldg(reinterpret_cast<const uint4*>(src + e0));
      } else if (n == 8 && (al & 7) == 0) {
        const uint2* s2 = reinterpret_cast<const uint2*>(src + e0);
        uint2* d2 = reinterpret_cast<uint2*>(dst + e0);
        d2[0] = __ldg(s2);
        d2[1] = __ldg(s2 + 1);
      } else {
        for (int e = 0; e < n; ++e) dst[e0 + e] = src[e0 + e];
      }
    }
  }
}

// dX[b, ih, iw, c..c+7] = relu'(X) * sum over the taps (kh, kw) that read the
// pixel of dcol[row(oh, ow), (kh, kw, c..c+7)], 8 channels per thread (C % 8 == 0).
// Only the taps congruent to the pixel modulo the stride are visited.
__global__ void col2im_kernel(const uint16_t* dcol, int64_t ldcol, const uint16_t* x_act, uint16_t* dx, ConvGeom g,
                              int relu) {
  const int cv = g.C / 8;
  const int per_image = g.H * g.W * cv;
  for (int b = blockIdx.y; b < g.B; b += gridDim.y) {
    const int64_t img = static_cast<int64_t>(b) * g.H * g.W * g.C;
    const uint16_t* db = dcol + static_cast<int64_t>(b) * g.OH * g.OW * ldcol;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < per_image; i += gridDim.x * blockDim.x) {
      const int v = i % cv;
      const int pix = i / cv;
      const int iw = pix % g.W, ih = pix / g.W;
      const int64_t off = img + static_cast<int64_t>(pix) * g.C + v * 8;
      uint4 mask = make_uint4(0xffffffffu, 0xffffffffu, 0xffffffffu, 0xffffffffu);
      if (relu) {
        const uint4 xa = __ldg(reinterpret_cast<const uint4*>(x_act + off));
        const uint32_t w4[4] = {xa.x, xa.y, xa.z, xa.w};
        uint32_t m4[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          // bf16 > 0: sign clear and non-zero magnitude, per half-word
          const uint32_t lo = (w4[q] & 0x8000u) == 0 && (w4[q] & 0x7fffu) != 0 ? 0x0000ffffu : 0u;
          const uint32_t hi = (w4[q] & 0x80000000u) == 0 && (w4[q] & 0x7fff0000u) != 0 ? 0xffff0000u : 0u;
          m4[q] = lo | hi;
        }
        mask = make_uint4(m4[0], m4[1], m4[2], m4[3]);
      }
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (mask.x | mask.y | mask.z | mask.w) {
        for (int kh = ih % g.S; kh < g.KH; kh += g.S) {
          const int oh = (ih - kh) / g.S;
          if (oh < 0) break;
          if (oh >= g.OH) continue;
          for (int kw = iw % g.S; kw < g.KW; kw += g.S) {
            const int ow = (iw - kw) / g.S;
            if (ow < 0) break;
            if (ow >= g.OW) continue;
            const uint4 d = __ldg(reinterpret_cast<const uint4*>(db + static_cast<int64_t>(oh * g.OW + ow) * ldcol +
                                                                 (kh * g.KW + kw) * g.C + v * 8));
            const uint32_t w4[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              acc[2 * q] += __uint_as_float(w4[q] << 16);
              acc[2 * q + 1] += __uint_as_float(w4[q] & 0xffff0000u);
            }
          }
        }
      }
      uint4 o;
      uint32_t* o4 = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        o4[q] = surfk::pack_bf16x2(acc[2 * q], acc[2 * q + 1]);
      o.x &= mask.x; o.y &= mask.y; o.z &= mask.z; o.w &= mask.w;
      *reinterpret_cast<uint4*>(dx + off) = o;
    }
  }
}

// out[n] += sum_m X[m, n] for bf16 X with N % 8 == 0 and 16-byte aligned rows:
// each thread owns one 8-column chunk of a row slot and accumulates in fp32.
__global__ void __launch_bounds__(256) colsum_vec_kernel(const uint16_t* x, int64_t ldx, int64_t M, int N,
                                                         float* out) {
  const int chunks = N / 8;
  const int slots = blockDim.x / chunks;          // rows in flight per block
  const int c = threadIdx.x % chunks, slot = threadIdx.x / chunks;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (slot < slots) {
    for (int64_t m = static_cast<int64_t>(blockIdx.x) * slots + slot; m < M;
         m += static_cast<int64_t>(gridDim.x) * slots) {
      const uint4 d = __ldg(reinterpret_cast<const uint4*>(x + m * ldx + c * 8));
      const uint32_t w4[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[2 * q] += __uint_as_float(w4[q] << 16);
        acc[2 * q + 1] += __uint_as_float(w4[q] & 0xffff0000u);
      }
    }
  }
  extern __shared__ float red[];                  // [blockDim.x][8]
#pragma unroll
  for (int e = 0; e < 8; ++e) red[threadIdx.x * 8 + e] = slot < slots ? acc[e] : 0.0f;
  __syncthreads();
  for (int j = threadIdx.x; j < N; j += blockDim.x) {
    const int cc = j / 8, e = j % 8;
    float s = 0.0f;
    for (int sl = 0; sl < slots; ++sl) s += red[(sl * chunks + cc) * 8 + e];
    atomicAdd(out + j, s);
  }
}

// out[n] += sum_m X[m, n] (X bf16 or fp32); 256 threads = 8 row groups x 32 columns
template <typename T>
__global__ void colsum_kernel(const T* x, int64_t ldx, int64_t M, int N, float* out) {
  const int col = blockIdx.x * 32 + (threadIdx.x & 31);
  const int grp = threadIdx.x >> 5;
  float acc = 0.0f;
  if (col < N) {
    for (int64_t m = blockIdx.y * 8 + grp; m < M; m += static_cast<int64_t>(gridDim.y) * 8) {
      if constexpr (sizeof(T) == 2) acc += surfk::bf16_to_f32(x[m * ldx + col]);
      else acc += x[m * ldx + col];
    }
  }
  __shared__ float red[8][32];
  red[grp][threadIdx.x & 31] = acc;
  __syncthreads();
  if (grp == 0 && col < N) {
    float s = 0.0f;
    for (int g = 0; g < 8; ++g) s += red[g][threadIdx.x];
    atomicAdd(out + col, s);
  }
}

// dst[i, :] = src[idx[i] + offset, :] for rows of `row_bytes` (multiple of 4).
// A source row outside [0, src_rows) is not read: the row is zeroed and the
// device error flag records kErrGatherIndex.
__global__ void gather_kernel(const uint8_t* src, int64_t src_stride, const int64_t* idx, int64_t offset, int64_t n,
                              int row_bytes, uint8_t* dst, int64_t dst_stride, int64_t src_rows, int* err) {
  const int words = row_bytes / 4;
  const int64_t total = n * words;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / words;
    const int w = static_cast<int>(i % words);
    const int64_t s = idx[r] + offset;
    uint32_t v = 0;
    if (s >= 0 && s < src_rows) v = reinterpret_cast<const uint32_t*>(src + s * src_stride)[w];
    else if (w == 0) surfk::report_error(err, surfk::kErrGatherIndex);
    reinterpret_cast<uint32_t*>(dst + r * dst_stride)[w] = v;
  }
}

// One warp per destination row, 16-byte vectors (rows, strides and bases
// 16-byte aligned): the index is read once per row and there is no
// per-element division; several vectors per lane are in flight.
__global__ void __launch_bounds__(256) gather16_kernel(const uint8_t* src, int64_t src_stride, const int64_t* idx,
                                                       int64_t offset, int64_t n, int row_bytes, uint8_t* dst,
                                                       int64_t dst_stride, int64_t src_rows, int* err) {
  const int lane = threadIdx.x & 31;
  const int vecs = row_bytes >> 4;
  const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t r = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5; r < n; r += warps) {
    const int64_t s = idx[r] + offset;
    const bool ok = s >= 0 && s < src_rows;
    if (!ok && lane == 0) surfk::report_error(err, surfk::kErrGatherIndex);
    const uint4* sp = reinterpret_cast<const uint4*>(src + (ok ? s : 0) * src_stride);
    uint4* dp = reinterpret_cast<uint4*>(dst + r * dst_stride);
#pragma unroll 4
    for (int c = lane; c < vecs; c += 32) dp[c] = ok ? __ldcs(sp + c) : make_uint4(0, 0, 0, 0);
  }
}

__global__ void f32_to_bf16_kernel(const float* x, int64_t ldx, uint16_t* y, int64_t ldy, int64_t rows, int cols) {
  const int64_t total = rows * cols;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols;
    const int c = static_cast<int>(i % cols);
    y[r * ldy + c] = surfk::f32_to_bf16(x[r * ldx + c]);
  }
}

// out[cls][c][a][b][co] = W[co][py + s*a][px + s*b][c], cls = py * s + px,
// a, b < k / s: the sub-kernels of the stride-s parity classes, transposed so
// that the input-gradient GEMM reads them K-major (K = (a, b, co)).
__global__ void conv_weight_t_kernel(const uint16_t* w, int CO, int C, int k, int s, uint16_t* out) {
  const int kt = k / s;
  const int per_cls = C * kt * kt * CO;
  const int total = s * s * per_cls;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int cls = i / per_cls;
    int r = i - cls * per_cls;
    const int c = r / (kt * kt * CO);
    r -= c * kt * kt * CO;
    const int a = r / (kt * CO);
    r -= a * kt * CO;
    const int b = r / CO, co = r - b * CO;
    const int kh = cls / s + s * a, kw = cls % s + s * b;
    out[i] = w[((static_cast<int64_t>(co) * k + kh) * k + kw) * C + c];
  }
}

int blocks_for(int64_t work, int threads) {
  const int64_t b = surfk::ceil_div(work, threads);
  return static_cast<int>(b < 1 ? 1 : (b > 148 * 64 ? 148 * 64 : b));
}

// Frame stacking (reference: python/train_fast.py:177-293, FrameRing and
// stack_from_buffer): decision t of env n sees its current frame and the
// frames of the decisions offs[1..K-1] before it, each reach-back clamped to
// the episode's age (the number of earlier decisions in the episode, capped at
// the deepest offset), so at a spawn every slot shows the spawn frame. Frames
// live slot-major in one buffer: frames[slot][env][ld], slot = pro + t in the
// trainer's rollout buffer (slots 0..pro-1 carry the previous rollout's last
// frames), or a ring of `ring` slots. The output row interleaves pixel-major:
// out[px][j][c] = frame_j[px][c] (frame index outer to the frame's own
// channels), the NHWC input of the first convolution.
struct StackArgs {
  const uint16_t* frames;   // bf16, slot 0
  int64_t slot_stride;      // elements between slots
  int ld;                   // elements between env rows of a slot
  int fr;                   // elements per frame (P * C0), multiple of 8
  int pro;                  // deepest offset (age cap)
  int ring;                 // > 0: slots are taken modulo ring
  int offs[8];              // offsets, newest (0) first
  int mode;                 // 0 rollout decision, 1 terminal (bootstrap), 2 minibatch gather
  int N;                    // envs per slot
  int lo;                   // mode 0: first env of the rows
  int slot0;                // modes 0/1: slot of the decision (mode 1: one past the newest stored)
  const float* done;        // mode 0: episode-ended flags of the previous decision, per row (NULL: keep ages)
  int* age_cur;             // modes 0/1: [N] running age
  int* age_rec;             // mode 0: ages recorded per row; mode 2: ages per flat sample (read)
  const int64_t* idx;       // mode 1: env per row; mode 2: flat sample t * N + n per row
  int64_t idx_bound;        // mode 2: flat samples stored (mode 1: N); an index outside is reported
  int* err;                 // device error flag (may be null)
  const uint16_t* cur;      // mode 1: the terminal frames, row r at cur + r * cur_ld
  int64_t cur_ld;
  uint16_t* out;
  int64_t out_ld;
};

template <int K, int C0>
__global__ void __launch_bounds__(256) frame_stack_kernel(StackArgs a) {
  __shared__ int s_age, s_env, s_slot, s_bad;
  const int r = blockIdx.x;
  if (threadIdx.x == 0) {
    int n = 0, age = 0, slot = 0;
    s_bad = 0;
    if (a.mode == 0) {
      n = a.lo + r;
      age = a.age_cur[n];
      if (a.done) age = a.done[r] != 0.0f ? 0 : min(age + 1, a.pro);
      a.age_cur[n] = age;
      a.age_rec[r] = age;
      slot = a.slot0;
    } else if (a.mode == 1) {
      const int64_t i = a.idx[r];
      if (i < 0 || i >= a.N) {
        s_bad = 1;
      } else {
        n = static_cast<int>(i);
        age = min(a.age_cur[n] + 1, a.pro);
        slot = a.slot0;
      }
    } else {
      const int64_t i = a.idx[r];
      if (i < 0 || i >= a.idx_bound) {
        s_bad = 1;
      } else {
        n = static_cast<int>(i % a.N);
        age = a.age_rec[i];
        slot = a.pro + static_cast<int>(i / a.N);
      }
    }
    if (s_bad) surfk::report_error(a.err, surfk::kErrStackIndex);
    s_age = age;
    s_env = n;
    s_slot = slot;
  }
  __syncthreads();
  if (s_bad) {                        // invalid index: the row is zeroed, nothing is read
    uint4* dst = reinterpret_cast<uint4*>(a.out + r * a.out_ld);
    for (int q = threadIdx.x; q < a.fr / 8 * K; q += blockDim.x) dst[q] = make_uint4(0, 0, 0, 0);
    return;
  }
  const int age = s_age, n = s_env, slot0 = s_slot;
  const uint4* src[K];
#pragma unroll
  for (int j = 0; j < K; ++j) {
    const int back = min(age, a.offs[j]);
    if (back == 0 && a.mode == 1) {
      src[j] = reinterpret_cast<const uint4*>(a.cur + r * a.cur_ld);
    } else {
      int sl = slot0 - back;
      if (a.ring > 0) sl = ((sl % a.ring) + a.ring) % a.ring;
      src[j] = reinterpret_cast<const uint4*>(a.frames + sl * a.slot_stride + static_cast<int64_t>(n) * a.ld);
    }
  }
  uint4* dst = reinterpret_cast<uint4*>(a.out + r * a.out_ld);
  const int chunks = a.fr / 8;
  for (int q = threadIdx.x; q < chunks; q += blockDim.x) {
    uint16_t in[K][8];
#pragma unroll
    for (int j = 0; j < K; ++j) *reinterpret_cast<uint4*>(in[j]) = __ldg(src[j] + q);
    // 8 frame elements = 8 / C0 pixels; their K frames form K output chunks
#pragma unroll
    for (int o8 = 0; o8 < K; ++o8) {
      uint16_t ov[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int o = o8 * 8 + e;
        const int px = o / (K * C0), j = (o / C0) % K, c = o % C0;
        ov[e] = in[j][px * C0 + c];
      }
      dst[q * K + o8] = *reinterpret_cast<const uint4*>(ov);
    }
  }
}

template <int C0>
int launch_stack(const StackArgs& a, int K, int rows, cudaStream_t s) {
  switch (K) {
    case 1: frame_stack_kernel<1, C0><<<rows, 256, 0, s>>>(a); break;
    case 2: frame_stack_kernel<2, C0><<<rows, 256, 0, s>>>(a); break;
    case 3: frame_stack_kernel<3, C0><<<rows, 256, 0, s>>>(a); break;
    case 4: frame_stack_kernel<4, C0><<<rows, 256, 0, s>>>(a); break;
    case 5: frame_stack_kernel<5, C0><<<rows, 256, 0, s>>>(a); break;
    default: return static_cast<int>(cudaErrorInvalidValue);
  }
  SURF_RETURN_LAUNCH();
}

}  // namespace

SURF_EXPORT int surf_im2col(const void* x, int B, int H, int W, int C, int KH, int KW, int S, void* col, int64_t ldcol,
                            void* stream) {
  ConvGeom g{B, H, W, C, KH, KW, S, (H - KH) / S + 1, (W - KW) / S + 1};
  const int per_image = g.OH * g.OW * KH * ((KW * C + 7) / 8);
  dim3 grid(static_cast<unsigned>(surfk::ceil_div(per_image, 256)), static_cast<unsigned>(B < 65535 ? B : 65535));
  im2col_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const uint16_t*>(x),
                                                                      static_cast<uint16_t*>(col), ldcol, g);
  SURF_RETURN_LAUNCH();
}

SURF_EXPORT int surf_col2im(const void* dcol, int64_t ldcol, const void* x_act, void* dx, int B, int H, int W, int C,
                            int KH, int KW, int S, int relu, void* stream) {
  ConvGeom g{B, H, W, C, KH, KW, S, (H - KH) / S + 1, (W - KW) / S + 1};
  if ((C & 7) || (ldcol & 7) || ((reinterpret_cast<uintptr_t>(dcol) | reinterpret_cast<uintptr_t>(dx) |
                                  reinterpret_cast<uintptr_t>(x_act)) & 15))
    return static_cast<int>(cudaErrorInvalidValue);     // 8-channel vectors need C % 8 == 0 and aligned rows
  const int per_image = H * W * (C / 8);
  dim3 grid(static_cast<unsigned>(surfk::ceil_div(per_image, 256)), static_cast<unsigned>(B < 65535 ? B : 65535));
  col2im_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(dcol), ldcol, static_cast<const uint16_t*>(x_act), static_cast<uint16_t*>(dx), g,
      relu);
  SURF_RETURN_LAUNCH();
}

// out (fp32 [N]) += column sums of X ([M, N], bf16 if bf16 != 0 else fp32)
SURF_EXPORT int surf_colsum(const void* x, int bf16, int64_t ldx, int64_t M, int N, float* out, void* stream) {
  auto s = static_cast<cudaStream_t>(stream);
  if (bf16 && N % 8 == 0 && N <= 2048 && ldx % 8 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    const int slots = 256 / (N / 8) > 0 ? 256 / (N / 8) : 1;
    const int threads = N / 8 > 256 ? N / 8 : 256;
    const int64_t want = surfk::ceil_div(M, static_cast<int64_t>(slots) * 16);
    const int blocks = static_cast<int>(want < 1 ? 1 : (want > 148 * 4 ? 148 * 4 : want));
    colsum_vec_kernel<<<blocks, threads, threads * 8 * sizeof(float), s>>>(static_cast<const uint16_t*>(x), ldx, M, N,
                                                                          out);
    SURF_RETURN_LAUNCH();
  }
  dim3 grid(static_cast<unsigned>((N + 31) / 32), static_cast<unsigned>(M / 64 > 256 ? 256 : (M / 64 < 1 ? 1 : M / 64)));
  if (bf16) colsum_kernel<uint16_t><<<grid, 256, 0, s>>>(static_cast<const uint16_t*>(x), ldx, M, N, out);
  else colsum_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(x), ldx, M, N, out);
  SURF_RETURN_LAUNCH();
}

// src_rows: rows of src (an index outside is reported through err, a device
// int the kernels set once; may be null).
SURF_EXPORT int surf_gather_rows(const void* src, int64_t src_stride_bytes, const int64_t* idx, int64_t offset,
                                 int64_t n, int row_bytes, void* dst, int64_t dst_stride_bytes, int64_t src_rows,
                                 int* err, void* stream) {
  if (row_bytes & 3) return static_cast<int>(cudaErrorInvalidValue);
  if (!((row_bytes | src_stride_bytes | dst_stride_bytes | reinterpret_cast<uintptr_t>(src) |
         reinterpret_cast<uintptr_t>(dst)) & 15) && row_bytes >= 512) {
    const int64_t blocks = surfk::ceil_div(n, 8);               // 8 rows (warps) per block
    gather16_kernel<<<static_cast<unsigned>(blocks < 148 * 16 ? blocks : 148 * 16), 256, 0,
                      static_cast<cudaStream_t>(stream)>>>(static_cast<const uint8_t*>(src), src_stride_bytes, idx,
                                                           offset, n, row_bytes, static_cast<uint8_t*>(dst),
                                                           dst_stride_bytes, src_rows, err);
    SURF_RETURN_LAUNCH();
  }
  gather_kernel<<<blocks_for(n * (row_bytes / 4), 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(src), src_stride_bytes, idx, offset, n, row_bytes, static_cast<uint8_t*>(dst),
      dst_stride_bytes, src_rows, err);
  SURF_RETURN_LAUNCH();
}

SURF_EXPORT int surf_f32_to_bf16(const float* x, int64_t ldx, void* y, int64_t ldy, int64_t rows, int cols, void* stream) {
  f32_to_bf16_kernel<<<blocks_for(rows * cols, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, ldx, static_cast<uint16_t*>(y), ldy, rows, cols);
  SURF_RETURN_LAUNCH();
}

// Sub-kernels of the stride-s parity classes for the implicit input gradient
// (see conv_weight_t_kernel); w: bf16 [CO, k, k, C]; out: bf16 [s*s, C, (k/s)^2 * CO].
SURF_EXPORT int surf_conv_weight_t(const void* w, int CO, int C, int k, int s, void* out, void* stream) {
  if (s < 1 || k % s) return static_cast<int>(cudaErrorInvalidValue);
  const int64_t total = static_cast<int64_t>(s) * s * C * (k / s) * (k / s) * CO;
  conv_weight_t_kernel<<<blocks_for(total, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(w), CO, C, k, s, static_cast<uint16_t*>(out));
  SURF_RETURN_LAUNCH();
}

// Build `rows` stacked policy inputs (see frame_stack_kernel). offs: K offsets
// (offs[0] == 0); every pointer row 16-byte aligned, fr % 8 == 0.
SURF_EXPORT int surf_frame_stack(const void* frames, int64_t slot_stride, int ld, int fr, int C0, int K,
                                 const int* offs, int pro, int ring, int mode, int N, int lo, int slot0,
                                 const float* done, int* age_cur, int* age_rec, const int64_t* idx, const void* cur,
                                 int64_t cur_ld, void* out, int64_t out_ld, int rows, int64_t idx_bound, int* err,
                                 void* stream) {
  if (K < 1 || K > 5 || (C0 != 1 && C0 != 2) || (fr & 7) || (ld & 7) || (slot_stride & 7) || (out_ld & 7) ||
      (cur_ld & 7) || mode < 0 || mode > 2 || pro < 0 || rows < 0 || N < 1 ||
      ((reinterpret_cast<uintptr_t>(frames) | reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(cur)) &
       15))
    return static_cast<int>(cudaErrorInvalidValue);
  if ((mode == 0 && (!age_cur || !age_rec)) || (mode == 1 && (!age_cur || !idx || !cur)) ||
      (mode == 2 && (!age_rec || !idx)))
    return static_cast<int>(cudaErrorInvalidValue);
  if (rows == 0) return 0;
  StackArgs a{};
  a.frames = static_cast<const uint16_t*>(frames);
  a.slot_stride = slot_stride;
  a.ld = ld;
  a.fr = fr;
  a.pro = pro;
  a.ring = ring;
  for (int j = 0; j < K; ++j) {
    if (offs[j] < 0 || offs[j] > pro) return static_cast<int>(cudaErrorInvalidValue);
    a.offs[j] = offs[j];
  }
  a.mode = mode;
  a.N = N;
  a.lo = lo;
  a.slot0 = slot0;
  a.done = done;
  a.age_cur = age_cur;
  a.age_rec = age_rec;
  a.idx_bound = mode == 1 ? N : idx_bound;
  a.err = err;
  a.idx = idx;
  a.cur = static_cast<const uint16_t*>(cur);
  a.cur_ld = cur_ld;
  a.out = static_cast<uint16_t*>(out);
  a.out_ld = out_ld;
  auto s = static_cast<cudaStream_t>(stream);
  return C0 == 1 ? launch_stack<1>(a, K, rows, s) : launch_stack<2>(a, K, rows, s);
}
