// Decode-time attention and KV-cache append for the generation engine.
//
// decode_attn: one new query token per sequence against that sequence's KV
// cache, GQA, head_dim 128.  Memory-bound (every cached K/V row is read once
// per step), so it is a split-K ("flash-decoding") CUDA-core kernel rather
// than a tensor-core one:
//   grid (splits, kv heads, sequences), 4 warps per CTA.  The CTA keeps the G
//   query heads of its kv head in shared memory (fp32); each warp takes 32
//   keys at a time, one key per lane: the lane reads its K row (16-byte
//   loads) and forms G dot products, the warp runs the online softmax per
//   head, then accumulates P V with each lane owning 4 of the 128 output
//   dims (V rows read coalesced, probabilities broadcast by shuffle).  Warps
//   merge in shared memory; splits write (acc, max, sum) partials that
//   decode_combine folds into the bf16 output.
// kv_append: writes the new token's rotated K and its V at position
// pos[b] of sequence b's cache rows.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "common.cuh"

namespace art {

namespace {
constexpr int DD = 128;
constexpr int MAXG = 16;
constexpr float kL2e = 1.4426950408889634f;
}  // namespace

__global__ void __launch_bounds__(128) decode_attn_kernel(
    const __nv_bfloat16* __restrict__ q, int64_t ldq, const __nv_bfloat16* __restrict__ kc,
    const __nv_bfloat16* __restrict__ vc, int64_t cache_seq_stride, int64_t cache_row_stride,
    const int* __restrict__ lens, float* __restrict__ part_acc, float* __restrict__ part_ml, int Hq, int Hkv,
    int nsplit, int chunk, int Lmax, float scale_log2) {
  const int split = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int G = Hq / Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ float sq[MAXG][DD];
  __shared__ float s_m[4][MAXG], s_l[4][MAXG];
  __shared__ float s_acc[4][MAXG][DD];

  for (int i = threadIdx.x; i < G * DD; i += 128) {
    const int g = i / DD, d = i % DD;
    sq[g][d] = bf2f(q[(int64_t)b * ldq + (int64_t)(hk * G + g) * DD + d]) * scale_log2;
  }
  __syncthreads();
  const int len = min(lens[b], Lmax);  // never read past the cache
  const int k_lo = split * chunk, k_hi = min(len, k_lo + chunk);
  float m[MAXG], l[MAXG], acc[MAXG][4];
#pragma unroll
  for (int g = 0; g < MAXG; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
    acc[g][0] = acc[g][1] = acc[g][2] = acc[g][3] = 0.f;
  }
  const __nv_bfloat16* kb = kc + (int64_t)b * cache_seq_stride + (int64_t)hk * DD;
  const __nv_bfloat16* vb = vc + (int64_t)b * cache_seq_stride + (int64_t)hk * DD;
  for (int j0 = k_lo + warp * 32; j0 < k_hi; j0 += 4 * 32) {
    const int j = j0 + lane;
    const bool valid = j < k_hi;
    float s[MAXG];
#pragma unroll
    for (int g = 0; g < MAXG; ++g) s[g] = 0.f;
    if (valid) {
      const uint4* krow = reinterpret_cast<const uint4*>(kb + (int64_t)j * cache_row_stride);
#pragma unroll 4
      for (int c = 0; c < DD / 8; ++c) {
        const uint4 u = __ldg(krow + c);
        const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
        float kf[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) kf[t] = bf2f(e[t]);
#pragma unroll
        for (int g = 0; g < MAXG; ++g) {
          if (g < G) {
#pragma unroll
            for (int t = 0; t < 8; ++t) s[g] += kf[t] * sq[g][c * 8 + t];
          }
        }
      }
    }
    // V slice of this lane for the 32 keys of the warp
#pragma unroll
    for (int g = 0; g < MAXG; ++g) {
      if (g >= G) continue;  // G is uniform: the whole warp takes the same branch
      const float x = valid ? s[g] : -INFINITY;
      const float mx = warp_max(x);
      const float m_new = fmaxf(m[g], mx);
      const float corr = (m[g] == -INFINITY) ? 0.f : exp2f(m[g] - m_new);
      const float p = valid ? exp2f(x - m_new) : 0.f;
      l[g] = l[g] * corr + warp_sum(p);
      m[g] = m_new;
      acc[g][0] *= corr;
      acc[g][1] *= corr;
      acc[g][2] *= corr;
      acc[g][3] *= corr;
      s[g] = p;
    }
    const int nk = min(32, k_hi - j0);
    for (int t = 0; t < nk; ++t) {
      const uint2 u = __ldg(reinterpret_cast<const uint2*>(vb + (int64_t)(j0 + t) * cache_row_stride) + lane);
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
      const float v0 = bf2f(e[0]), v1 = bf2f(e[1]), v2 = bf2f(e[2]), v3 = bf2f(e[3]);
#pragma unroll
      for (int g = 0; g < MAXG; ++g) {
        if (g < G) {
          const float p = __shfl_sync(0xffffffffu, s[g], t);
          acc[g][0] += p * v0;
          acc[g][1] += p * v1;
          acc[g][2] += p * v2;
          acc[g][3] += p * v3;
        }
      }
    }
  }
  // merge the 4 warps
#pragma unroll
  for (int g = 0; g < MAXG; ++g) {
    if (g >= G) continue;
    if (lane == 0) {
      s_m[warp][g] = m[g];
      s_l[warp][g] = l[g];
    }
    s_acc[warp][g][lane * 4 + 0] = acc[g][0];
    s_acc[warp][g][lane * 4 + 1] = acc[g][1];
    s_acc[warp][g][lane * 4 + 2] = acc[g][2];
    s_acc[warp][g][lane * 4 + 3] = acc[g][3];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * DD; i += 128) {
    const int g = i / DD, d = i % DD;
    float M = -INFINITY;
    for (int w = 0; w < 4; ++w) M = fmaxf(M, s_m[w][g]);
    float L = 0.f, A = 0.f;
    for (int w = 0; w < 4; ++w) {
      if (s_m[w][g] == -INFINITY) continue;
      const float c = exp2f(s_m[w][g] - M);
      L += s_l[w][g] * c;
      A += s_acc[w][g][d] * c;
    }
    const int64_t slot = ((int64_t)b * Hq + hk * G + g) * nsplit + split;
    part_acc[slot * DD + d] = A;
    if (d == 0) {
      part_ml[slot * 2 + 0] = M;
      part_ml[slot * 2 + 1] = L;
    }
  }
}

__global__ void decode_combine_kernel(const float* __restrict__ part_acc, const float* __restrict__ part_ml,
                                      __nv_bfloat16* __restrict__ o, int64_t ldo, int Hq, int nsplit) {
  const int bh = blockIdx.x;  // b * Hq + h
  const int d = threadIdx.x;  // 128 threads
  const int b = bh / Hq, h = bh % Hq;
  float M = -INFINITY;
  for (int s = 0; s < nsplit; ++s) M = fmaxf(M, part_ml[((int64_t)bh * nsplit + s) * 2]);
  float L = 0.f, A = 0.f;
  for (int s = 0; s < nsplit; ++s) {
    const int64_t slot = (int64_t)bh * nsplit + s;
    const float ms = part_ml[slot * 2];
    if (ms == -INFINITY) continue;
    const float c = exp2f(ms - M);
    L += part_ml[slot * 2 + 1] * c;
    A += part_acc[slot * DD + d] * c;
  }
  o[(int64_t)b * ldo + (int64_t)h * DD + d] = f2bf(L > 0.f ? A / L : 0.f);
}

// q [B, Hq, 128] (row stride free, heads packed); caches [B, Lmax, Hkv, 128]
// contiguous; lens [B] int32 = keys visible to each sequence's new token.
torch::Tensor decode_attn(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor lens,
                          double scale) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kBFloat16 && q.dim() == 3 && q.size(2) == DD);
  TORCH_CHECK(q.stride(2) == 1 && q.stride(1) == DD && q.stride(0) % 8 == 0);
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous() && k_cache.dim() == 4 && k_cache.size(3) == DD);
  TORCH_CHECK(k_cache.sizes() == v_cache.sizes() && k_cache.scalar_type() == at::kBFloat16);
  TORCH_CHECK(lens.scalar_type() == at::kInt && lens.is_contiguous());
  const int64_t B = q.size(0), Hq = q.size(1), Lmax = k_cache.size(1), Hkv = k_cache.size(2);
  TORCH_CHECK(k_cache.size(0) >= B && lens.numel() == B && Hq % Hkv == 0 && Hq / Hkv <= MAXG);
  auto o = torch::empty({B, Hq, DD}, q.options());
  if (B == 0) return o;
  int sms = 148;
  int dev = 0;
  ART_CUDA_CHECK(cudaGetDevice(&dev));
  ART_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  int nsplit = (int)std::max<int64_t>(1, (2 * sms + B * Hkv - 1) / (B * Hkv));
  nsplit = (int)std::min<int64_t>(nsplit, (Lmax + 127) / 128);
  const int chunk = (int)(((Lmax + nsplit - 1) / nsplit + 31) / 32 * 32);
  auto part_acc = torch::empty({B * Hq * nsplit * DD}, q.options().dtype(at::kFloat));
  auto part_ml = torch::empty({B * Hq * nsplit * 2}, q.options().dtype(at::kFloat));
  auto stream = at::cuda::getCurrentCUDAStream();
  decode_attn_kernel<<<dim3(nsplit, Hkv, B), 128, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), q.stride(0),
      reinterpret_cast<const __nv_bfloat16*>(k_cache.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(v_cache.data_ptr()), k_cache.stride(0), k_cache.stride(1),
      lens.data_ptr<int>(), part_acc.data_ptr<float>(), part_ml.data_ptr<float>(), (int)Hq, (int)Hkv, nsplit, chunk,
      (int)Lmax, (float)(scale * kL2e));
  ART_CUDA_CHECK(cudaGetLastError());
  decode_combine_kernel<<<(unsigned)(B * Hq), DD, 0, stream>>>(part_acc.data_ptr<float>(), part_ml.data_ptr<float>(),
                                                            reinterpret_cast<__nv_bfloat16*>(o.data_ptr()), o.stride(0),
                                                            (int)Hq, nsplit);
  ART_CUDA_CHECK(cudaGetLastError());
  return o;
}

__global__ void kv_append_kernel(const __nv_bfloat16* __restrict__ k, int64_t ldk,
                                 const __nv_bfloat16* __restrict__ v, int64_t ldv, const int* __restrict__ slot,
                                 const int* __restrict__ pos, __nv_bfloat16* __restrict__ kc,
                                 __nv_bfloat16* __restrict__ vc, int64_t seq_stride, int64_t row_stride, int width) {
  const int b = blockIdx.x;
  const int64_t dst = (int64_t)slot[b] * seq_stride + (int64_t)pos[b] * row_stride;
  for (int i = threadIdx.x; i < width / 8; i += blockDim.x) {
    reinterpret_cast<uint4*>(kc + dst)[i] = reinterpret_cast<const uint4*>(k + (int64_t)b * ldk)[i];
    reinterpret_cast<uint4*>(vc + dst)[i] = reinterpret_cast<const uint4*>(v + (int64_t)b * ldv)[i];
  }
}

// Row b of k/v ([n, Hkv*128] views) goes to cache row pos[b] of cache sequence slot[b].
void kv_append(torch::Tensor k, torch::Tensor v, torch::Tensor slot, torch::Tensor pos, torch::Tensor k_cache,
               torch::Tensor v_cache) {
  TORCH_CHECK(k.dim() == 2 && v.dim() == 2 && k.stride(1) == 1 && v.stride(1) == 1);
  TORCH_CHECK(k.scalar_type() == at::kBFloat16 && k_cache.scalar_type() == at::kBFloat16 && k_cache.is_contiguous() &&
              v_cache.is_contiguous());
  const int64_t n = k.size(0), width = k.size(1);
  TORCH_CHECK(width == k_cache.size(2) * k_cache.size(3) && width % 8 == 0 && k.stride(0) % 8 == 0 &&
              v.stride(0) % 8 == 0);
  TORCH_CHECK(slot.numel() == n && pos.numel() == n && slot.scalar_type() == at::kInt && pos.scalar_type() == at::kInt);
  if (n == 0) return;
  kv_append_kernel<<<(unsigned)n, 64, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(k.data_ptr()), k.stride(0),
      reinterpret_cast<const __nv_bfloat16*>(v.data_ptr()), v.stride(0), slot.data_ptr<int>(), pos.data_ptr<int>(),
      reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr()), reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr()),
      k_cache.stride(0), k_cache.stride(1), (int)width);
  ART_CUDA_CHECK(cudaGetLastError());
}

}  // namespace art
