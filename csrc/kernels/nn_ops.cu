// nn_ops.cu — the non-GEMM layers of the policy network (sm_100a).
//
//   * im2col: NHWC bf16 activations -> convolution patch rows (kh, kw, c order)
//     so that a convolution is one tensor-core GEMM;
//   * col2im_relu: the transposed scatter, written as a gather (no atomics),
//     fused with the ReLU derivative of the layer below;
//   * colsum: bias gradients (sum of dY over rows), fp32 accumulation;
//   * gather_rows: minibatch rows of the rollout buffers (any element size);
//   * cast kernels between fp32 and bf16.
#include <cstdint>

#include "surf_cuda.cuh"

namespace {

struct ConvGeom {
  int B, H, W, C;      // input NHWC
  int KH, KW, S;       // kernel, stride (no padding)
  int OH, OW;
};

// one thread per (output row, kh, 8-element chunk of the kw*C run)
__global__ void im2col_kernel(const uint16_t* x, uint16_t* col, int64_t ldcol, ConvGeom g) {
  const int run = g.KW * g.C;                 // contiguous elements per kh
  const int chunks = (run + 7) / 8;
  const int64_t total = static_cast<int64_t>(g.B) * g.OH * g.OW * g.KH * chunks;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int ch = static_cast<int>(i % chunks);
    int64_t r = i / chunks;
    const int kh = static_cast<int>(r % g.KH);
    const int64_t row = r / g.KH;
    const int ow = static_cast<int>(row % g.OW);
    const int64_t t = row / g.OW;
    const int oh = static_cast<int>(t % g.OH);
    const int b = static_cast<int>(t / g.OH);
    const int ih = oh * g.S + kh, iw = ow * g.S;
    const uint16_t* src = x + ((static_cast<int64_t>(b) * g.H + ih) * g.W + iw) * g.C;
    uint16_t* dst = col + row * ldcol + kh * run;
    const int e0 = ch * 8;
    const int n = min(8, run - e0);
    if (n == 8 && ((reinterpret_cast<uintptr_t>(src + e0) | reinterpret_cast<uintptr_t>(dst + e0)) & 15) == 0) {
      *reinterpret_cast<uint4*>(dst + e0) = *reinterpret_cast<const uint4*>(src + e0);
    } else if (n == 8 && ((reinterpret_cast<uintptr_t>(src + e0) | reinterpret_cast<uintptr_t>(dst + e0)) & 3) == 0) {
      const uint32_t* s4 = reinterpret_cast<const uint32_t*>(src + e0);
      uint32_t* d4 = reinterpret_cast<uint32_t*>(dst + e0);
      d4[0] = s4[0]; d4[1] = s4[1]; d4[2] = s4[2]; d4[3] = s4[3];
    } else {
      for (int e = 0; e < n; ++e) dst[e0 + e] = src[e0 + e];
    }
  }
}

// dX[b, ih, iw, c] = relu'(X) * sum over the (kh, kw) taps that read it of dcol
__global__ void col2im_kernel(const uint16_t* dcol, int64_t ldcol, const uint16_t* x_act, uint16_t* dx, ConvGeom g,
                              int relu) {
  const int64_t total = static_cast<int64_t>(g.B) * g.H * g.W * g.C;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % g.C);
    int64_t t = i / g.C;
    const int iw = static_cast<int>(t % g.W);
    t /= g.W;
    const int ih = static_cast<int>(t % g.H);
    const int b = static_cast<int>(t / g.H);
    float acc = 0.0f;
    if (!relu || surfk::bf16_to_f32(x_act[i]) > 0.0f) {
      for (int kh = 0; kh < g.KH; ++kh) {
        const int oh_s = ih - kh;
        if (oh_s < 0 || oh_s % g.S) continue;
        const int oh = oh_s / g.S;
        if (oh >= g.OH) continue;
        for (int kw = 0; kw < g.KW; ++kw) {
          const int ow_s = iw - kw;
          if (ow_s < 0 || ow_s % g.S) continue;
          const int ow = ow_s / g.S;
          if (ow >= g.OW) continue;
          const int64_t row = (static_cast<int64_t>(b) * g.OH + oh) * g.OW + ow;
          acc += surfk::bf16_to_f32(dcol[row * ldcol + (kh * g.KW + kw) * g.C + c]);
        }
      }
    }
    dx[i] = surfk::f32_to_bf16(acc);
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

// dst[i, :] = src[idx[i] + offset, :] for rows of `row_bytes` (multiple of 4)
__global__ void gather_kernel(const uint8_t* src, int64_t src_stride, const int64_t* idx, int64_t offset, int64_t n,
                              int row_bytes, uint8_t* dst, int64_t dst_stride) {
  const int words = row_bytes / 4;
  const int64_t total = n * words;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / words;
    const int w = static_cast<int>(i % words);
    const int64_t s = idx[r] + offset;
    reinterpret_cast<uint32_t*>(dst + r * dst_stride)[w] = reinterpret_cast<const uint32_t*>(src + s * src_stride)[w];
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

int blocks_for(int64_t work, int threads) {
  const int64_t b = surfk::ceil_div(work, threads);
  return static_cast<int>(b < 1 ? 1 : (b > 148 * 64 ? 148 * 64 : b));
}

}  // namespace

SURF_EXPORT int surf_im2col(const void* x, int B, int H, int W, int C, int KH, int KW, int S, void* col, int64_t ldcol,
                            void* stream) {
  ConvGeom g{B, H, W, C, KH, KW, S, (H - KH) / S + 1, (W - KW) / S + 1};
  const int64_t work = static_cast<int64_t>(B) * g.OH * g.OW * KH * ((KW * C + 7) / 8);
  im2col_kernel<<<blocks_for(work, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(x), static_cast<uint16_t*>(col), ldcol, g);
  SURF_RETURN_LAUNCH();
}

SURF_EXPORT int surf_col2im(const void* dcol, int64_t ldcol, const void* x_act, void* dx, int B, int H, int W, int C,
                            int KH, int KW, int S, int relu, void* stream) {
  ConvGeom g{B, H, W, C, KH, KW, S, (H - KH) / S + 1, (W - KW) / S + 1};
  const int64_t work = static_cast<int64_t>(B) * H * W * C;
  col2im_kernel<<<blocks_for(work, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(dcol), ldcol, static_cast<const uint16_t*>(x_act), static_cast<uint16_t*>(dx), g,
      relu);
  SURF_RETURN_LAUNCH();
}

// out (fp32 [N]) += column sums of X ([M, N], bf16 if bf16 != 0 else fp32)
SURF_EXPORT int surf_colsum(const void* x, int bf16, int64_t ldx, int64_t M, int N, float* out, void* stream) {
  dim3 grid(static_cast<unsigned>((N + 31) / 32), static_cast<unsigned>(M / 64 > 256 ? 256 : (M / 64 < 1 ? 1 : M / 64)));
  auto s = static_cast<cudaStream_t>(stream);
  if (bf16) colsum_kernel<uint16_t><<<grid, 256, 0, s>>>(static_cast<const uint16_t*>(x), ldx, M, N, out);
  else colsum_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(x), ldx, M, N, out);
  SURF_RETURN_LAUNCH();
}

SURF_EXPORT int surf_gather_rows(const void* src, int64_t src_stride_bytes, const int64_t* idx, int64_t offset,
                                 int64_t n, int row_bytes, void* dst, int64_t dst_stride_bytes, void* stream) {
  if (row_bytes & 3) return static_cast<int>(cudaErrorInvalidValue);
  gather_kernel<<<blocks_for(n * (row_bytes / 4), 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(src), src_stride_bytes, idx, offset, n, row_bytes, static_cast<uint8_t*>(dst),
      dst_stride_bytes);
  SURF_RETURN_LAUNCH();
}

SURF_EXPORT int surf_f32_to_bf16(const float* x, int64_t ldx, void* y, int64_t ldy, int64_t rows, int cols, void* stream) {
  f32_to_bf16_kernel<<<blocks_for(rows * cols, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, ldx, static_cast<uint16_t*>(y), ldy, rows, cols);
  SURF_RETURN_LAUNCH();
}
