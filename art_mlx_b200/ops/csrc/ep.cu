// Expert-parallel token exchange over peer memory (NVLink P2P stores).
//
// scatter_rows: row i of `src` [n, H] (optionally scaled by `scale[i]`) is
//   stored into row dst_row[i] of the buffer of rank dst_rank[i]; the buffer
//   bases come from a per-rank pointer table (own rank = local pointer).
//   One warp per row, 16-byte vector stores.  With a one-entry table it is a
//   local permutation (single GPU).
// combine_rows: y[t] = sum_j w[t, j] * slots[t * k + j]  (fp32 accumulate).
// segment_offsets: device-side exclusive prefix sums for the routing plan.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "common.cuh"

namespace art {

__global__ void scatter_rows_kernel(const __nv_bfloat16* __restrict__ src, int64_t n, int H,
                                    const int64_t* __restrict__ src_idx,
                                    const int* __restrict__ dst_rank, const int64_t* __restrict__ dst_row,
                                    const float* __restrict__ scale, const int64_t* __restrict__ bases,
                                    int64_t ld_dst, const int64_t* __restrict__ dst_limit) {
  const int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= n) return;
  const int r = dst_rank ? dst_rank[w] : 0;
  const int64_t row = dst_row[w];
  if (row < 0 || (dst_limit && row >= dst_limit[0])) return;  // dropped (over capacity)
  __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(bases[r]) + row * ld_dst;
  const __nv_bfloat16* s = src + (src_idx ? src_idx[w] : w) * H;
  const float sc = scale ? scale[w] : 1.f;
  for (int c = lane * 8; c < H; c += 256) {
    uint4 v = *reinterpret_cast<const uint4*>(s + c);
    if (scale) {
      __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&v);
#pragma unroll
      for (int k = 0; k < 8; ++k) e[k] = f2bf(bf2f(e[k]) * sc);
    }
    *reinterpret_cast<uint4*>(dst + c) = v;
  }
}

__global__ void combine_rows_kernel(const __nv_bfloat16* __restrict__ slots, const float* __restrict__ w,
                                    int64_t T, int k, int H, __nv_bfloat16* __restrict__ out) {
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  for (int c = lane * 8; c < H; c += 256) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int j = 0; j < k; ++j) {
      const float wj = w ? w[t * k + j] : 1.f;
      uint4 v = *reinterpret_cast<const uint4*>(slots + (t * k + j) * H + c);
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] += wj * bf2f(e[q]);
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + t * H + c) = o;
  }
}

// gather_rows: dst[i] = scale[i] * rows[src_row[i]] of rank src_rank[i] (peer loads).
__global__ void gather_rows_kernel(__nv_bfloat16* __restrict__ dst, int64_t n, int H,
                                   const int* __restrict__ src_rank, const int64_t* __restrict__ src_row,
                                   const float* __restrict__ scale, const int64_t* __restrict__ bases,
                                   int64_t ld_src) {
  const int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= n) return;
  const int r = src_rank ? src_rank[w] : 0;
  const int64_t row = src_row[w];
  __nv_bfloat16* d = dst + w * H;
  if (row < 0) {
    for (int c = lane * 8; c < H; c += 256) *reinterpret_cast<uint4*>(d + c) = make_uint4(0, 0, 0, 0);
    return;
  }
  const __nv_bfloat16* s = reinterpret_cast<const __nv_bfloat16*>(bases[r]) + row * ld_src;
  const float sc = scale ? scale[w] : 1.f;
  for (int c = lane * 8; c < H; c += 256) {
    uint4 v = *reinterpret_cast<const uint4*>(s + c);
    if (scale) {
      __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&v);
#pragma unroll
      for (int k = 0; k < 8; ++k) e[k] = f2bf(bf2f(e[k]) * sc);
    }
    *reinterpret_cast<uint4*>(d + c) = v;
  }
}

void gather_rows(torch::Tensor dst, c10::optional<torch::Tensor> src_rank, torch::Tensor src_row,
                 c10::optional<torch::Tensor> scale, torch::Tensor bases, int64_t ld_src) {
  TORCH_CHECK(dst.is_contiguous() && dst.scalar_type() == at::kBFloat16 && dst.dim() == 2);
  const int64_t n = dst.size(0);
  const int H = dst.size(1);
  TORCH_CHECK(H % 8 == 0 && ld_src % 8 == 0 && src_row.numel() == n);
  if (n == 0) return;
  gather_rows_kernel<<<(n + 7) / 8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(dst.data_ptr()), n, H,
      src_rank.has_value() ? src_rank->data_ptr<int>() : nullptr, src_row.data_ptr<int64_t>(),
      scale.has_value() ? scale->data_ptr<float>() : nullptr, bases.data_ptr<int64_t>(), ld_src);
  ART_CUDA_CHECK(cudaGetLastError());
}

static void scatter_impl(torch::Tensor src, int64_t n, const int64_t* src_idx,
                         c10::optional<torch::Tensor> dst_rank, torch::Tensor dst_row,
                         c10::optional<torch::Tensor> scale, torch::Tensor bases, int64_t ld_dst,
                         c10::optional<torch::Tensor> dst_limit) {
  TORCH_CHECK(src.is_contiguous() && src.scalar_type() == at::kBFloat16 && src.dim() == 2);
  const int H = src.size(1);
  TORCH_CHECK(H % 8 == 0 && ld_dst % 8 == 0);
  TORCH_CHECK(dst_row.scalar_type() == at::kLong && dst_row.numel() == n);
  if (scale.has_value()) TORCH_CHECK(scale->scalar_type() == at::kFloat && scale->numel() == n && scale->is_contiguous());
  if (n == 0) return;
  scatter_rows_kernel<<<(n + 7) / 8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(src.data_ptr()), n, H, src_idx,
      dst_rank.has_value() ? dst_rank->data_ptr<int>() : nullptr, dst_row.data_ptr<int64_t>(),
      scale.has_value() ? scale->data_ptr<float>() : nullptr, bases.data_ptr<int64_t>(), ld_dst,
      dst_limit.has_value() ? dst_limit->data_ptr<int64_t>() : nullptr);
  ART_CUDA_CHECK(cudaGetLastError());
}

void scatter_rows(torch::Tensor src, c10::optional<torch::Tensor> dst_rank, torch::Tensor dst_row,
                  c10::optional<torch::Tensor> scale, torch::Tensor bases, int64_t ld_dst,
                  c10::optional<torch::Tensor> dst_limit) {
  scatter_impl(src, src.size(0), nullptr, dst_rank, dst_row, scale, bases, ld_dst, dst_limit);
}

// Row i of the transfer is src[src_idx[i]] (e.g. a token repeated for each of its k slots).
void scatter_rows_idx(torch::Tensor src, torch::Tensor src_idx, torch::Tensor dst_rank, torch::Tensor dst_row,
                      c10::optional<torch::Tensor> scale, torch::Tensor bases, int64_t ld_dst) {
  TORCH_CHECK(src_idx.scalar_type() == at::kLong && src_idx.is_contiguous());
  TORCH_CHECK(dst_rank.scalar_type() == at::kInt && dst_rank.is_contiguous());
  scatter_impl(src, src_idx.numel(), src_idx.data_ptr<int64_t>(), dst_rank, dst_row, scale, bases, ld_dst,
               c10::nullopt);
}

torch::Tensor combine_rows(torch::Tensor slots, c10::optional<torch::Tensor> w, int64_t k) {
  TORCH_CHECK(slots.is_contiguous() && slots.scalar_type() == at::kBFloat16);
  const int H = slots.size(1);
  const int64_t T = slots.size(0) / k;
  auto out = torch::empty({T, H}, slots.options());
  if (T == 0) return out;
  combine_rows_kernel<<<(T + 7) / 8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(slots.data_ptr()), w.has_value() ? w->data_ptr<float>() : nullptr,
      T, (int)k, H, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  ART_CUDA_CHECK(cudaGetLastError());
  return out;
}

}  // namespace art
