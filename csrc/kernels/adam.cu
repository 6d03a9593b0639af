// adam.cu — global-norm gradient clipping fused with the Adam update (sm_100a).
//
// All policy parameters live in one flat fp32 master buffer with a flat fp32
// gradient buffer beside it (the backward GEMMs accumulate straight into
// views of it), plus a bf16 copy that the forward/backward GEMMs read.
// One optimizer step is two kernels on the stream:
//   surf_adam_norm   sum of squared gradients (fp64 accumulator), step += 1
//   surf_adam_update coef = min(1, max_norm / (||g|| + 1e-6)); Adam with bias
//                    correction (torch.optim.Adam semantics, eps outside the
//                    bias-corrected square root); writes the fp32 master, the
//                    bf16 copy and zeroes the gradient for the next minibatch.
// Hyper-parameters are read from device memory (lr, betas, eps, max_norm,
// step) so a CUDA graph of the update sees schedule changes.
// Reference behaviour: nn.utils.clip_grad_norm_(…, 0.5) + torch.optim.Adam
// (eps 1e-5, fused), python/train_fast.py:1505-1506, 2194-2195.
#include <cstdint>

#include "surf_cuda.cuh"

namespace {

struct Hyper { float lr, beta1, beta2, eps, max_norm, step; };

__global__ void norm_kernel(const float* g, int64_t n, double* acc, Hyper* h) {
  double s = 0.0;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float v = g[i];
    s += static_cast<double>(v) * v;
  }
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  __shared__ double red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += red[w];
    atomicAdd(acc, t);
    if (blockIdx.x == 0) h->step += 1.0f;
  }
}

__global__ void update_kernel(float* p, float* g, float* m, float* v, uint16_t* p_bf16, int64_t n, const double* acc,
                              const Hyper* h) {
  const float norm = static_cast<float>(sqrt(*acc));
  const float coef = h->max_norm > 0.0f ? fminf(1.0f, h->max_norm / (norm + 1e-6f)) : 1.0f;
  const float b1 = h->beta1, b2 = h->beta2, t = h->step;
  const float bc1 = 1.0f - powf(b1, t), bc2 = 1.0f - powf(b2, t);
  const float step = h->lr / bc1;
  const float rbc2 = rsqrtf(bc2);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float gi = g[i] * coef;
    const float mi = b1 * m[i] + (1.0f - b1) * gi;
    const float vi = b2 * v[i] + (1.0f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    const float pi = p[i] - step * mi / (sqrtf(vi) * rbc2 + h->eps);
    p[i] = pi;
    if (p_bf16) p_bf16[i] = surfk::f32_to_bf16(pi);
    g[i] = 0.0f;
  }
}

int blocks(int64_t n) {
  const int64_t b = surfk::ceil_div(n, 256);
  return static_cast<int>(b < 1 ? 1 : (b > 148 * 8 ? 148 * 8 : b));
}

}  // namespace

// acc: one fp64 zeroed by the caller before this launch; hyper: 6 floats.
SURF_EXPORT int surf_adam_norm(const float* g, int64_t n, double* acc, float* hyper, void* stream) {
  norm_kernel<<<blocks(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(g, n, acc, reinterpret_cast<Hyper*>(hyper));
  SURF_RETURN_LAUNCH();
}

SURF_EXPORT int surf_adam_update(float* p, float* g, float* m, float* v, void* p_bf16, int64_t n, const double* acc,
                                 const float* hyper, void* stream) {
  update_kernel<<<blocks(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(p, g, m, v, static_cast<uint16_t*>(p_bf16), n,
                                                                           acc, reinterpret_cast<const Hyper*>(hyper));
  SURF_RETURN_LAUNCH();
}
