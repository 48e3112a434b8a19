// Flat-buffer AdamW for the LoRA parameters.
//
// All trainable LoRA tensors live in one contiguous fp32 master buffer with a
// bf16 compute copy, one fp32 gradient buffer and the two moment buffers, so
// the whole optimizer step is two launches: a sum-of-squares reduction for the
// global grad norm (written to device memory, no host sync) and one fused
// update that applies loss scaling, norm clipping, bias-corrected AdamW with
// decoupled weight decay, writes the bf16 copy and zeroes the gradient.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "common.cuh"

namespace art {

__global__ void sumsq_kernel(const float* __restrict__ g, int64_t n, float* __restrict__ out) {
  __shared__ float red[32];
  float acc = 0.f;
  const int64_t n4 = n / 4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 v = reinterpret_cast<const float4*>(g)[i];
    acc += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  for (int64_t i = n4 * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    acc += g[i] * g[i];
  acc = block_sum(acc, red);
  if (threadIdx.x == 0) atomicAdd(out, acc);
}

// hp: [0]=lr, [1]=beta1, [2]=beta2, [3]=eps, [4]=weight_decay, [5]=max_grad_norm (<=0: off),
//     [6]=grad_scale (e.g. 1/num_tokens), [7]=step (1-based, for bias correction)
// norm_sq: device scalar, sum of squares of the *unscaled* gradient.
__global__ void adamw_kernel(float* __restrict__ p, __nv_bfloat16* __restrict__ p16,
                             float* __restrict__ g, float* __restrict__ m, float* __restrict__ v,
                             int64_t n, const float* __restrict__ hp,
                             const float* __restrict__ norm_sq, float* __restrict__ norm_out) {
  const float lr = hp[0], b1 = hp[1], b2 = hp[2], eps = hp[3], wd = hp[4], clip = hp[5];
  const float gs = hp[6], step = hp[7];
  const float gnorm = sqrtf(*norm_sq) * gs;
  float coef = gs;
  if (clip > 0.f && gnorm > clip) coef *= clip / (gnorm + 1e-6f);
  if (norm_out && blockIdx.x == 0 && threadIdx.x == 0) *norm_out = gnorm;
  const float bc1 = 1.f - powf(b1, step), bc2 = 1.f - powf(b2, step);
  const float step_size = lr / bc1;
  const float inv_bc2_sqrt = rsqrtf(bc2);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float gi = g[i] * coef;
    const float mi = b1 * m[i] + (1.f - b1) * gi;
    const float vi = b2 * v[i] + (1.f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    float pi = p[i] * (1.f - lr * wd);
    pi -= step_size * mi / (sqrtf(vi) * inv_bc2_sqrt + eps);
    p[i] = pi;
    p16[i] = f2bf(pi);
    g[i] = 0.f;
  }
}

static int grid_for(int64_t n, int threads) {
  int64_t b = (n + threads - 1) / threads;
  if (b > 148 * 8) b = 148 * 8;
  return (int)(b < 1 ? 1 : b);
}

torch::Tensor grad_sumsq(torch::Tensor g) {
  TORCH_CHECK(g.is_contiguous() && g.scalar_type() == at::kFloat);
  auto out = torch::zeros({1}, g.options());
  sumsq_kernel<<<grid_for(g.numel() / 4 + 1, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      g.data_ptr<float>(), g.numel(), out.data_ptr<float>());
  ART_CUDA_CHECK(cudaGetLastError());
  return out;
}

void adamw_step(torch::Tensor p, torch::Tensor p16, torch::Tensor g, torch::Tensor m,
                torch::Tensor v, torch::Tensor hp, torch::Tensor norm_sq, torch::Tensor norm_out) {
  TORCH_CHECK(p.is_contiguous() && g.is_contiguous() && m.is_contiguous() && v.is_contiguous());
  TORCH_CHECK(p16.scalar_type() == at::kBFloat16 && p16.numel() == p.numel());
  const int64_t n = p.numel();
  adamw_kernel<<<grid_for(n, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      p.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(p16.data_ptr()), g.data_ptr<float>(),
      m.data_ptr<float>(), v.data_ptr<float>(), n, hp.data_ptr<float>(), norm_sq.data_ptr<float>(),
      norm_out.data_ptr<float>());
  ART_CUDA_CHECK(cudaGetLastError());
}

}  // namespace art
