// adam.cu — global-norm gradient clipping fused with the Adam update (sm_100a).
//
// All policy parameters live in one flat fp32 master buffer with a flat fp32
// gradient buffer beside it (the backward GEMMs accumulate straight into
// views of it), plus a bf16 copy that the forward/backward GEMMs read.
// One optimizer step is two kernels on the stream:
//   surf_adam_norm   sum of squared gradients: per-block fp64 partials, the
//                    last block to finish adds them in block order (the norm
//                    does not depend on block timing) into acc[0]; step += 1
//   surf_adam_update coef = min(1, max_norm / (||g|| + 1e-6)); Adam with bias
//                    correction (torch.optim.Adam semantics, eps outside the
//                    bias-corrected square root); writes the fp32 master, the
//                    bf16 copy and zeroes the gradient for the next minibatch.
// Both stream 16-byte vectors (4 parameters per thread and step).
// Hyper-parameters are read from device memory (lr, betas, eps, max_norm,
// step) so a CUDA graph of the update sees schedule changes.
// Reference behaviour: nn.utils.clip_grad_norm_(…, 0.5) + torch.optim.Adam
// (eps 1e-5, fused), python/train_fast.py:1505-1506, 2194-2195.
#include <cstdint>

#include "surf_cuda.cuh"

namespace {

struct Hyper { float lr, beta1, beta2, eps, max_norm, step; };

constexpr int kNormBlocks = 296;         // partials in acc[2 .. 2 + kNormBlocks)

// acc[0]: the squared norm (written by the last block); acc[1]: arrival
// counter (its bits as an unsigned int; zero between launches); acc[2..]:
// per-block partial sums.
__global__ void __launch_bounds__(256) norm_kernel(const float* g, int64_t n, double* acc, Hyper* h) {
  double s = 0.0;
  const int64_t n4 = n >> 2;
  const float4* g4 = reinterpret_cast<const float4*>(g);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float4 v = g4[i];
    s += static_cast<double>(v.x) * v.x + static_cast<double>(v.y) * v.y + static_cast<double>(v.z) * v.z +
         static_cast<double>(v.w) * v.w;
  }
  if (blockIdx.x == 0)
    for (int64_t i = (n4 << 2) + threadIdx.x; i < n; i += blockDim.x) s += static_cast<double>(g[i]) * g[i];
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  __shared__ double red[8];
  __shared__ bool last;
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += red[w];
    acc[2 + blockIdx.x] = t;
    __threadfence();
    unsigned int* cnt = reinterpret_cast<unsigned int*>(acc + 1);
    last = atomicAdd(cnt, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (threadIdx.x < 32) {
    // fixed order: lane l adds partials l, l + 32, ..., then a fixed tree
    double t = 0.0;
    for (int b = threadIdx.x; b < static_cast<int>(gridDim.x); b += 32) t += __ldcg(acc + 2 + b);
    for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) {
      acc[0] = t;
      *reinterpret_cast<unsigned int*>(acc + 1) = 0u;
      h->step += 1.0f;
    }
  }
}

__device__ __forceinline__ void adam_one(float& p, float& m, float& v, float g, float coef, float b1, float b2,
                                         float step, float rbc2, float eps) {
  const float gi = g * coef;
  m = b1 * m + (1.0f - b1) * gi;
  v = b2 * v + (1.0f - b2) * gi * gi;
  p = p - step * m / (sqrtf(v) * rbc2 + eps);
}

__global__ void __launch_bounds__(256) update_kernel(float* p, float* g, float* m, float* v, uint16_t* p_bf16,
                                                     int64_t n, const double* acc, const Hyper* h) {
  const float norm = static_cast<float>(sqrt(*acc));
  const float coef = h->max_norm > 0.0f ? fminf(1.0f, h->max_norm / (norm + 1e-6f)) : 1.0f;
  const float b1 = h->beta1, b2 = h->beta2, t = h->step;
  const float bc1 = 1.0f - powf(b1, t), bc2 = 1.0f - powf(b2, t);
  const float step = h->lr / bc1;
  const float rbc2 = rsqrtf(bc2);
  const float eps = h->eps;
  const int64_t n4 = n >> 2;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float4 pp = reinterpret_cast<float4*>(p)[i];
    float4 mm = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    const float4 gg = reinterpret_cast<float4*>(g)[i];
    adam_one(pp.x, mm.x, vv.x, gg.x, coef, b1, b2, step, rbc2, eps);
    adam_one(pp.y, mm.y, vv.y, gg.y, coef, b1, b2, step, rbc2, eps);
    adam_one(pp.z, mm.z, vv.z, gg.z, coef, b1, b2, step, rbc2, eps);
    adam_one(pp.w, mm.w, vv.w, gg.w, coef, b1, b2, step, rbc2, eps);
    reinterpret_cast<float4*>(p)[i] = pp;
    reinterpret_cast<float4*>(m)[i] = mm;
    reinterpret_cast<float4*>(v)[i] = vv;
    reinterpret_cast<float4*>(g)[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (p_bf16)
      reinterpret_cast<uint2*>(p_bf16)[i] = make_uint2(
          static_cast<uint32_t>(surfk::f32_to_bf16(pp.x)) | static_cast<uint32_t>(surfk::f32_to_bf16(pp.y)) << 16,
          static_cast<uint32_t>(surfk::f32_to_bf16(pp.z)) | static_cast<uint32_t>(surfk::f32_to_bf16(pp.w)) << 16);
  }
  if (blockIdx.x == 0) {
    for (int64_t i = (n4 << 2) + threadIdx.x; i < n; i += blockDim.x) {
      float pi = p[i], mi = m[i], vi = v[i];
      adam_one(pi, mi, vi, g[i], coef, b1, b2, step, rbc2, eps);
      p[i] = pi;
      m[i] = mi;
      v[i] = vi;
      if (p_bf16) p_bf16[i] = surfk::f32_to_bf16(pi);
      g[i] = 0.0f;
    }
  }
}

int blocks(int64_t n) {
  const int64_t b = surfk::ceil_div(n, 1024);              // one float4 per thread
  return static_cast<int>(b < 1 ? 1 : (b > 148 * 16 ? 148 * 16 : b));
}

}  // namespace

// acc: 2 + 296 fp64 (see norm_kernel), zeroed once at allocation and left
// ready by every launch; hyper: 6 floats. All buffers 16-byte aligned.
SURF_EXPORT int surf_adam_norm(const float* g, int64_t n, double* acc, float* hyper, void* stream) {
  if (reinterpret_cast<uintptr_t>(g) & 15) return static_cast<int>(cudaErrorInvalidValue);
  norm_kernel<<<kNormBlocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(g, n, acc, reinterpret_cast<Hyper*>(hyper));
  SURF_RETURN_LAUNCH();
}

SURF_EXPORT int surf_adam_acc_size() { return 2 + kNormBlocks; }

SURF_EXPORT int surf_adam_update(float* p, float* g, float* m, float* v, void* p_bf16, int64_t n, const double* acc,
                                 const float* hyper, void* stream) {
  if ((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(m) |
       reinterpret_cast<uintptr_t>(v)) & 15 || (reinterpret_cast<uintptr_t>(p_bf16) & 7))
    return static_cast<int>(cudaErrorInvalidValue);
  update_kernel<<<blocks(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(p, g, m, v, static_cast<uint16_t*>(p_bf16), n,
                                                                           acc, reinterpret_cast<const Hyper*>(hyper));
  SURF_RETURN_LAUNCH();
}
