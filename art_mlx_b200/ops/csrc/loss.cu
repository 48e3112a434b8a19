// LM-head log-softmax statistics and gradient over the vocabulary, and the
// fused GRPO/CISPO/PPO token-loss (value and d loss / d logprob).
//
// logits_stats: one CTA per row of a [T, V] bf16 logits chunk; computes, in one
//   pass with an online max rescaling, lse = log sum exp(x), the target logit
//   and the entropy H = lse - sum softmax(x) * x.
// logits_grad_: in place, dlogits = g * (onehot(target) - softmax(x)).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "common.cuh"

namespace art {

struct SoftmaxAcc {
  float m, s, sx;  // running max, sum exp(x - m), sum exp(x - m) * x
};

__device__ __forceinline__ SoftmaxAcc sm_merge(SoftmaxAcc a, SoftmaxAcc b) {
  if (a.m == -INFINITY) return b;
  if (b.m == -INFINITY) return a;
  const float m = fmaxf(a.m, b.m);
  const float ea = __expf(a.m - m), eb = __expf(b.m - m);
  return {m, a.s * ea + b.s * eb, a.sx * ea + b.sx * eb};
}

__global__ void logits_stats_kernel(const __nv_bfloat16* __restrict__ logits, int64_t ld, int V,
                                    const int64_t* __restrict__ targets, float* __restrict__ lse,
                                    float* __restrict__ tgt, float* __restrict__ ent) {
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* x = logits + row * ld;
  SoftmaxAcc acc{-INFINITY, 0.f, 0.f};
  // vectorised main loop (V multiple of 8 is required by the host wrapper)
  for (int c = threadIdx.x * 8; c < V; c += blockDim.x * 8) {
    uint4 v = *reinterpret_cast<const uint4*>(x + c);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
    float f[8];
    float mloc = acc.m;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      f[k] = bf2f(e[k]);
      mloc = fmaxf(mloc, f[k]);
    }
    const float scale = (acc.m == -INFINITY) ? 0.f : __expf(acc.m - mloc);
    float s = acc.s * scale, sx = acc.sx * scale;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float p = __expf(f[k] - mloc);
      s += p;
      sx += p * f[k];
    }
    acc = {mloc, s, sx};
  }
  // warp merge
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    SoftmaxAcc other{__shfl_xor_sync(0xffffffffu, acc.m, o), __shfl_xor_sync(0xffffffffu, acc.s, o),
                     __shfl_xor_sync(0xffffffffu, acc.sx, o)};
    acc = sm_merge(acc, other);
  }
  __shared__ SoftmaxAcc red[32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) red[wid] = acc;
  __syncthreads();
  if (wid == 0) {
    const int nw = blockDim.x >> 5;
    acc = lane < nw ? red[lane] : SoftmaxAcc{-INFINITY, 0.f, 0.f};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      SoftmaxAcc other{__shfl_xor_sync(0xffffffffu, acc.m, o),
                       __shfl_xor_sync(0xffffffffu, acc.s, o),
                       __shfl_xor_sync(0xffffffffu, acc.sx, o)};
      acc = sm_merge(acc, other);
    }
    if (lane == 0) {
      const float l = acc.m + logf(acc.s);
      lse[row] = l;
      if (ent) ent[row] = l - acc.sx / acc.s;
      const int64_t t = targets[row];
      tgt[row] = (t >= 0 && t < V) ? bf2f(x[t]) : 0.f;
    }
  }
}

__global__ void logits_grad_kernel(__nv_bfloat16* __restrict__ logits, int64_t ld, int V,
                                   const int64_t* __restrict__ targets,
                                   const float* __restrict__ lse, const float* __restrict__ g) {
  const int64_t row = blockIdx.x;
  const float gr = g[row];
  __nv_bfloat16* x = logits + row * ld;
  const int64_t t = targets[row];
  if (gr == 0.f) {
    for (int c = threadIdx.x * 8; c < V; c += blockDim.x * 8)
      *reinterpret_cast<uint4*>(x + c) = make_uint4(0, 0, 0, 0);
    return;
  }
  const float l = lse[row];
  for (int c = threadIdx.x * 8; c < V; c += blockDim.x * 8) {
    uint4 v = *reinterpret_cast<const uint4*>(x + c);
    __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&v);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float p = __expf(bf2f(e[k]) - l);
      e[k] = f2bf(gr * (((c + k) == t ? 1.f : 0.f) - p));
    }
    *reinterpret_cast<uint4*>(x + c) = v;
  }
}

std::vector<torch::Tensor> logits_stats(torch::Tensor logits, torch::Tensor targets, bool entropy) {
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1 && logits.scalar_type() == at::kBFloat16);
  TORCH_CHECK(targets.scalar_type() == at::kLong && targets.is_contiguous());
  const int64_t T = logits.size(0);
  const int V = logits.size(1);
  TORCH_CHECK(V % 8 == 0 && logits.stride(0) % 8 == 0, "vocab must be a multiple of 8");
  auto opts = logits.options().dtype(at::kFloat);
  auto lse = torch::empty({T}, opts), tgt = torch::empty({T}, opts);
  auto ent = entropy ? torch::empty({T}, opts) : torch::Tensor();
  if (T > 0)
    logits_stats_kernel<<<T, 512, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), logits.stride(0), V,
        targets.data_ptr<int64_t>(), lse.data_ptr<float>(), tgt.data_ptr<float>(),
        entropy ? ent.data_ptr<float>() : nullptr);
  ART_CUDA_CHECK(cudaGetLastError());
  return {lse, tgt, ent};
}

void logits_grad_(torch::Tensor logits, torch::Tensor targets, torch::Tensor lse, torch::Tensor g) {
  const int64_t T = logits.size(0);
  const int V = logits.size(1);
  TORCH_CHECK(g.scalar_type() == at::kFloat && g.is_contiguous() && lse.is_contiguous());
  if (T > 0)
    logits_grad_kernel<<<T, 512, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), logits.stride(0), V,
        targets.data_ptr<int64_t>(), lse.data_ptr<float>(), g.data_ptr<float>());
  ART_CUDA_CHECK(cudaGetLastError());
}

// ----------------------------------------------------------------------------
// GRPO token loss, token-level importance ratio.  Inputs are aligned (column t
// scores token t+1).  Two launches: (1) masked KL sum + mask count, (2) per
// token loss and gradient.  The reduction denominator is applied on device.
// cfg: [0]=ppo, [1]=eps, [2]=eps_hi, [3]=kl_coef, [4]=kl_source_sample,
//      [5]=tis_upper(0=off), [6]=mask_prob_ratio, [7]=kimi_tau, [8]=max_neg_is(0=off),
//      [9]=denominator (>0 explicit, <0 masked mean, 0 sum), [10]=T
// ----------------------------------------------------------------------------
__global__ void grpo_stats_kernel(const float* __restrict__ newlp, const float* __restrict__ oldlp,
                                  const float* __restrict__ reflp, const float* __restrict__ mask,
                                  int64_t T, const float* __restrict__ cfg, float* __restrict__ sums) {
  __shared__ float red[32];
  const bool kl_sample = cfg[4] != 0.f;
  float kl = 0.f, cnt = 0.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < T;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float m = mask[i];
    cnt += m;
    if (reflp) {
      float o = oldlp[i];
      if (isnan(o)) o = newlp[i];
      const float src = kl_sample ? o : newlp[i];
      kl += (src - reflp[i]) * m;
    }
  }
  kl = block_sum(kl, red);
  cnt = block_sum(cnt, red);
  if (threadIdx.x == 0) {
    atomicAdd(&sums[0], kl);
    atomicAdd(&sums[1], cnt);
  }
}

__global__ void grpo_loss_kernel(const float* __restrict__ newlp, const float* __restrict__ oldlp,
                                 const float* __restrict__ adv, const float* __restrict__ w,
                                 const float* __restrict__ mask, const float* __restrict__ reflp,
                                 const float* __restrict__ origlp, const float* __restrict__ cfg,
                                 const float* __restrict__ sums, float* __restrict__ grad,
                                 float* __restrict__ out) {
  __shared__ float red[32];
  const int64_t T = (int64_t)cfg[10];
  const bool ppo = cfg[0] != 0.f;
  const float eps = cfg[1], eps_hi = cfg[2], kl_coef = cfg[3];
  const bool kl_sample = cfg[4] != 0.f;
  const float tis = cfg[5];
  const bool mpr = cfg[6] != 0.f;
  const float tau = cfg[7], cap = cfg[8];
  // cfg[9]: >0 explicit denominator; <0 masked-token mean; 0 plain sum
  const float denom = cfg[9] > 0.f ? cfg[9] : (cfg[9] < 0.f ? sums[1] + 1e-18f : 1.f);
  const float avg_kl = sums[0] / (sums[1] + 1e-18f);
  float lsum = 0.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < T;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float m = mask[i];
    const float nl = newlp[i];
    float ol = oldlp[i];
    if (isnan(ol)) ol = nl;
    const float d = nl - ol;
    float r = __expf(d);
    if (cap > 0.f) r = fminf(r, cap);
    if (mpr) r = (r > 1.f - eps && r < 1.f + eps_hi) ? r : 0.f;
    float a = adv[i];
    if (tau != 0.f) a -= tau * d;
    if (kl_coef > 0.f && reflp) {
      const float src = kl_sample ? ol : nl;
      const float klt = (src - reflp[i]) * m;
      a += kl_coef * (avg_kl - klt) * m;
    }
    const float rc = fminf(fmaxf(r, 1.f - eps), 1.f + eps_hi);
    float loss, g;
    // r carries gradient d r / d newlp = r unless it was capped or zeroed
    const bool capped = cap > 0.f && __expf(d) > cap;
    const bool zeroed = mpr && r == 0.f;
    const float dr = (capped || zeroed) ? 0.f : r;
    if (ppo) {
      // -min(r*a, clip(r)*a); inside the clip range both branches agree
      const float u = r * a, v = rc * a;
      const bool inside = r >= 1.f - eps && r <= 1.f + eps_hi;
      if (inside || u < v) {
        loss = -u;
        g = -a * dr;
      } else {
        loss = -v;
        g = 0.f;
      }
    } else {
      loss = -rc * a * nl;
      g = -rc * a;
    }
    if (tis > 0.f) {
      float tr = r;
      if (origlp) {
        float og = origlp[i];
        if (isnan(og)) og = nl;
        tr = __expf(ol - og);
      }
      const float f = fminf(tr, tis);
      loss *= f;
      g *= f;
    }
    const float s = w[i] * m;
    loss *= s;
    grad[i] = g * s / denom;
    lsum += loss;
  }
  lsum = block_sum(lsum, red);
  if (threadIdx.x == 0) atomicAdd(&out[0], lsum);
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    out[1] = denom;
    out[2] = avg_kl;
  }
}

// Returns (grad [T] = d(loss_reduced)/d newlp, out [3] = {loss_sum, denom, avg_kl}).
std::vector<torch::Tensor> grpo_token_loss(torch::Tensor newlp, torch::Tensor oldlp,
                                           torch::Tensor adv, torch::Tensor w, torch::Tensor mask,
                                           c10::optional<torch::Tensor> reflp,
                                           c10::optional<torch::Tensor> origlp,
                                           torch::Tensor cfg) {
  const int64_t T = newlp.numel();
  auto opts = newlp.options();
  auto sums = torch::zeros({2}, opts);
  auto out = torch::zeros({3}, opts);
  auto grad = torch::empty_like(newlp);
  const int threads = 256;
  int blocks = (int)std::min<int64_t>((T + threads - 1) / threads, 148 * 4);
  if (blocks < 1) blocks = 1;
  const float* rp = reflp.has_value() ? reflp->data_ptr<float>() : nullptr;
  const float* op = origlp.has_value() ? origlp->data_ptr<float>() : nullptr;
  auto stream = at::cuda::getCurrentCUDAStream();
  grpo_stats_kernel<<<blocks, threads, 0, stream>>>(newlp.data_ptr<float>(), oldlp.data_ptr<float>(),
                                                    rp, mask.data_ptr<float>(), T,
                                                    cfg.data_ptr<float>(), sums.data_ptr<float>());
  grpo_loss_kernel<<<blocks, threads, 0, stream>>>(
      newlp.data_ptr<float>(), oldlp.data_ptr<float>(), adv.data_ptr<float>(), w.data_ptr<float>(),
      mask.data_ptr<float>(), rp, op, cfg.data_ptr<float>(), sums.data_ptr<float>(),
      grad.data_ptr<float>(), out.data_ptr<float>());
  ART_CUDA_CHECK(cudaGetLastError());
  return {grad, out};
}

}  // namespace art
