// Low-rank (LoRA) side products over row segments, sm_100a.
//
// The adapter's products are skinny: one side is the rank r (8..64) and the
// other a hidden or intermediate size, so they are bound by the read of the
// big operand, not by tensor-core throughput.  Two kernels cover every one
// of them, for one dense segment (a linear layer) or many (one per MoE
// expert, rows laid out expert-contiguous):
//
//   lowrank_rows:  Y[n, :R] = scale[n] * X[src[n], :K] @ W_g^T        (W_g: R x K)
//                  x A^T (u), dy B (the rank-side input gradient), with an
//                  optional row gather (token -> slot) and per-row scale
//                  (routing weights);
//   lowrank_wgrad: G_g(r, c) += alpha * sum_{n in g} P[n, r] * Q[n, c]
//                  dA = s dyB^T x  and  dB^T = s u^T dy  (fp32 accumulate,
//                  G addressed through strides so dB lands in its [C, R]
//                  layout).
//
// Both run on the warp-level tensor-core path (mma.sync m16n8k16, bf16 in,
// fp32 accumulate): each CTA stages a 64-wide k-slice of its operands in
// shared memory with cp.async (double-buffered), so the big operand is read
// once per CTA.  Reference counterpart: the grouped varlen LoRA GEMMs of
// src/art/megatron/kernels/cute_grouped_lora_quack.py:257-680 (x A_e then
// (.) B_e with cu_seqlens over expert token offsets; dA/dB over cu_seqlens_k).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "common.cuh"

namespace art {

namespace {
constexpr int LR_ROWS = 64;  // rows per CTA (4 warps x 16)
constexpr int LR_KC = 64;    // k-slice per stage
constexpr int LR_LD = LR_KC + 8;  // padded smem row (elements): conflict-free ldmatrix
}  // namespace

// grid: one CTA per (segment, 64-row block), from `blocks` [nb] = (segment, row0).
template <int R>
__global__ void __launch_bounds__(128) lowrank_rows_kernel(
    const __nv_bfloat16* __restrict__ X, int64_t ldx, const int64_t* __restrict__ src,
    const float* __restrict__ scale, const int* __restrict__ seg_off, const int* __restrict__ seg_group,
    const int2* __restrict__ blocks, const __nv_bfloat16* __restrict__ W, int64_t w_gs, int64_t w_rs,
    int64_t w_ks, int K, __nv_bfloat16* __restrict__ Y, int64_t ldy) {
  __shared__ __align__(16) __nv_bfloat16 sX[2][LR_ROWS * LR_LD];
  __shared__ __align__(16) __nv_bfloat16 sW[2][R * LR_LD];
  const int2 blk = blocks[blockIdx.x];
  const int seg = blk.x;
  const int n0 = blk.y, n_end = seg_off[seg + 1];
  const __nv_bfloat16* Wg = W + (int64_t)seg_group[seg] * w_gs;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool w_contig = (w_ks == 1) && ((w_rs & 7) == 0) && ((reinterpret_cast<uintptr_t>(Wg) & 15) == 0);

  auto stage = [&](int kc, int buf) {
    // X rows (gathered): 64 rows x 64 k = 512 chunks of 16 B
    for (int c = tid; c < LR_ROWS * (LR_KC / 8); c += 128) {
      const int r = c >> 3, ch = c & 7;
      const int n = n0 + r;
      const int k = kc + ch * 8;
      const bool ok = n < n_end && k < K;
      const int64_t row = ok ? (src ? src[n] : n) : 0;
      cp_async16(smem_u32(&sX[buf][r * LR_LD + ch * 8]), X + row * ldx + (ok ? k : 0), ok ? 16 : 0);
    }
    // W_g slice: R rows x 64 k
    if (w_contig) {
      for (int c = tid; c < R * (LR_KC / 8); c += 128) {
        const int r = c >> 3, ch = c & 7;
        const int k = kc + ch * 8;
        const bool ok = k < K;
        cp_async16(smem_u32(&sW[buf][r * LR_LD + ch * 8]), Wg + r * w_rs + (ok ? k : 0), ok ? 16 : 0);
      }
    } else {
      for (int c = tid; c < R * LR_KC; c += 128) {
        const int r = c / LR_KC, kk = c % LR_KC;
        const int k = kc + kk;
        sW[buf][r * LR_LD + kk] = k < K ? Wg[r * w_rs + (int64_t)k * w_ks] : __float2bfloat16(0.f);
      }
    }
  };

  float acc[R / 8][4];
#pragma unroll
  for (int j = 0; j < R / 8; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[j][e] = 0.f;

  const int nkc = (K + LR_KC - 1) / LR_KC;
  stage(0, 0);
  cp_async_commit();
  for (int it = 0; it < nkc; ++it) {
    const int buf = it & 1;
    if (it + 1 < nkc) stage((it + 1) * LR_KC, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < LR_KC / 16; ++kk) {
      uint32_t a[4];
      ldsm_x4(a, smem_u32(&sX[buf][(warp * 16 + (lane & 15)) * LR_LD + kk * 16 + (lane >> 4) * 8]));
#pragma unroll
      for (int j = 0; j < R / 16; ++j) {
        uint32_t b[4];
        // rows n = j*16 + (lane & 7) + ((lane >> 4) << 3) of W, k halves by (lane >> 3) & 1
        ldsm_x4(b, smem_u32(&sW[buf][(j * 16 + (lane & 7) + ((lane >> 4) << 3)) * LR_LD + kk * 16 +
                                     ((lane >> 3) & 1) * 8]));
        mma16816(acc[2 * j], a, b[0], b[1]);
        mma16816(acc[2 * j + 1], a, b[2], b[3]);
      }
      if constexpr (R % 16 == 8) {
        uint32_t b[2];
        const int j = R / 16;
        // 8 rows of W: x2 load
        const uint32_t addr = smem_u32(&sW[buf][(j * 16 + (lane & 7)) * LR_LD + kk * 16 + ((lane >> 3) & 1) * 8]);
        asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n" : "=r"(b[0]), "=r"(b[1]) : "r"(addr));
        mma16816(acc[2 * j], a, b[0], b[1]);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();
  // write: thread holds rows (lane>>2) and +8, columns 2*(lane&3) (+1) of each n-tile
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int n = n0 + warp * 16 + (lane >> 2) + h * 8;
    if (n >= n_end) continue;
    const float sc = scale ? scale[n] : 1.f;
#pragma unroll
    for (int j = 0; j < R / 8; ++j) {
      const int col = j * 8 + 2 * (lane & 3);
      *reinterpret_cast<uint32_t*>(Y + (int64_t)n * ldy + col) = pack_bf16x2(acc[j][2 * h] * sc, acc[j][2 * h + 1] * sc);
    }
  }
}

// grid: (segment, row split) blocks from `blocks` [nb] = (segment, split) x column chunks of 128.
// G_g(r, c) += alpha * sum_n P[n, r] Q[n, c]; rows of segment s split into
// `splits` contiguous parts, one per CTA (fp32 atomic adds into G).
template <int R>
__global__ void __launch_bounds__(128) lowrank_wgrad_kernel(
    const __nv_bfloat16* __restrict__ P, int64_t ldp, const __nv_bfloat16* __restrict__ Q, int64_t ldq,
    const int* __restrict__ seg_off, const int* __restrict__ seg_group, const int2* __restrict__ blocks, int splits,
    int C, float* __restrict__ G, int64_t g_gs, int64_t g_rs, int64_t g_cs, float alpha) {
  constexpr int RP = (R + 15) / 16 * 16;  // M padded to the mma tile
  constexpr int CW = 128;              // columns per CTA (4 warps x 32)
  constexpr int NK = 32;               // rows per stage
  __shared__ __align__(16) __nv_bfloat16 sP[2][NK * (RP + 8)];
  __shared__ __align__(16) __nv_bfloat16 sQ[2][NK * (CW + 8)];
  const int2 blk = blocks[blockIdx.x];
  const int seg = blk.x, part = blk.y;
  const int c0 = blockIdx.y * CW;
  const int s0 = seg_off[seg], s1 = seg_off[seg + 1];
  const int len = s1 - s0;
  const int per = (len + splits - 1) / splits;
  const int r0 = s0 + part * per, r1 = min(s1, r0 + per);
  if (r0 >= r1) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int PLD = RP + 8, QLD = CW + 8;

  auto stage = [&](int n0, int buf) {
    // P: NK rows x RP cols (zero pad rows past the end and columns past R)
    for (int c = tid; c < NK * (RP / 8); c += 128) {
      const int r = c / (RP / 8), ch = c % (RP / 8);
      const int n = n0 + r;
      const bool ok = n < r1 && ch * 8 < R;
      cp_async16(smem_u32(&sP[buf][r * PLD + ch * 8]), P + (ok ? (int64_t)n * ldp + ch * 8 : 0), ok ? 16 : 0);
    }
    for (int c = tid; c < NK * (CW / 8); c += 128) {
      const int r = c / (CW / 8), ch = c % (CW / 8);
      const int n = n0 + r;
      const int col = c0 + ch * 8;
      const bool ok = n < r1 && col < C;
      cp_async16(smem_u32(&sQ[buf][r * QLD + ch * 8]), Q + (ok ? (int64_t)n * ldq + col : 0), ok ? 16 : 0);
    }
  };

  float acc[RP / 16][4][4];
#pragma unroll
  for (int m = 0; m < RP / 16; ++m)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[m][j][e] = 0.f;

  const int nst = (r1 - r0 + NK - 1) / NK;
  stage(r0, 0);
  cp_async_commit();
  for (int it = 0; it < nst; ++it) {
    const int buf = it & 1;
    if (it + 1 < nst) stage(r0 + (it + 1) * NK, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
#pragma unroll
    for (int ks = 0; ks < NK / 16; ++ks) {
      // B fragments (k = rows n, n = columns c): Q is [n][c] (c contiguous) -> transposed load
      uint32_t b[4][2];
#pragma unroll
      for (int j2 = 0; j2 < 2; ++j2) {
        uint32_t t[4];
        const int krow = ks * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int col = warp * 32 + j2 * 16 + (lane >> 4) * 8;
        ldsm_x4_t(t, smem_u32(&sQ[buf][krow * QLD + col]));
        b[2 * j2][0] = t[0];
        b[2 * j2][1] = t[1];
        b[2 * j2 + 1][0] = t[2];
        b[2 * j2 + 1][1] = t[3];
      }
#pragma unroll
      for (int m = 0; m < RP / 16; ++m) {
        // A fragment (m = rank r, k = rows n): P is [n][r] -> transposed load
        uint32_t a[4];
        const int mi = lane >> 3;
        const int krow = ks * 16 + (lane & 7) + ((mi >> 1) << 3);
        const int rc = m * 16 + ((mi & 1) << 3);
        ldsm_x4_t(a, smem_u32(&sP[buf][krow * PLD + rc]));
#pragma unroll
        for (int j = 0; j < 4; ++j) mma16816(acc[m][j], a, b[j][0], b[j][1]);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();
#pragma unroll
  for (int m = 0; m < RP / 16; ++m)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = m * 16 + (lane >> 2) + h * 8;
      if (r >= R) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = c0 + warp * 32 + j * 8 + 2 * (lane & 3);
        float* g = G + (int64_t)seg_group[seg] * g_gs + (int64_t)r * g_rs;
        if (c < C) atomicAdd(g + (int64_t)c * g_cs, alpha * acc[m][j][2 * h]);
        if (c + 1 < C) atomicAdd(g + (int64_t)(c + 1) * g_cs, alpha * acc[m][j][2 * h + 1]);
      }
    }
}

// ---------------------------------------------------------------- host side
static torch::Tensor to_dev_i32(const std::vector<int32_t>& v, const torch::Device& dev) {
  auto h = torch::from_blob(const_cast<int32_t*>(v.data()), {(int64_t)v.size()}, torch::kInt32).pin_memory();
  return h.to(dev, /*non_blocking=*/true);
}

// Y [N, R] = scale * X[src] @ W_g^T per segment.  seg_off: host offsets
// (segments cover rows [0, N)); seg_group: host group index per segment;
// w: bf16 tensor addressed as w_gs * g + w_rs * r + w_ks * k (elements).
torch::Tensor lowrank_rows(torch::Tensor x, c10::optional<torch::Tensor> src, c10::optional<torch::Tensor> scale,
                           std::vector<int64_t> seg_off, std::vector<int64_t> seg_group, torch::Tensor w,
                           int64_t R, int64_t w_gs, int64_t w_rs, int64_t w_ks, int64_t K,
                           c10::optional<torch::Tensor> out) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1);
  TORCH_CHECK(x.stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0, "x rows 16-byte aligned");
  TORCH_CHECK(w.is_cuda() && w.scalar_type() == at::kBFloat16);
  TORCH_CHECK(K % 8 == 0 && K <= x.size(1), "K must be a multiple of 8 within x");
  TORCH_CHECK(R == 8 || R == 16 || R == 24 || R == 32 || R == 48 || R == 64 || R == 96,
              "rank width 8/16/24/32/48/64/96");
  const int64_t S = (int64_t)seg_group.size();
  TORCH_CHECK((int64_t)seg_off.size() == S + 1 && seg_off[0] == 0);
  const int64_t N = seg_off[S];
  if (src.has_value()) {
    TORCH_CHECK(src->scalar_type() == at::kLong && src->numel() >= N && src->is_contiguous());
  } else {
    TORCH_CHECK(x.size(0) >= N);
  }
  if (scale.has_value()) TORCH_CHECK(scale->scalar_type() == at::kFloat && scale->numel() >= N && scale->is_contiguous());
  torch::Tensor y;
  if (out.has_value()) {
    y = *out;
    TORCH_CHECK(y.scalar_type() == at::kBFloat16 && y.size(0) >= N && y.size(1) == R && y.stride(1) == 1 &&
                y.stride(0) % 2 == 0);
  } else {
    y = torch::empty({N, R}, x.options());
  }
  if (N == 0) return y;
  std::vector<int32_t> off(S + 1), grp(S), blk;
  for (int64_t s = 0; s <= S; ++s) off[s] = (int32_t)seg_off[s];
  for (int64_t s = 0; s < S; ++s) {
    TORCH_CHECK(seg_off[s + 1] >= seg_off[s], "segment offsets must be non-decreasing");
    grp[s] = (int32_t)seg_group[s];
    for (int64_t r0 = seg_off[s]; r0 < seg_off[s + 1]; r0 += LR_ROWS) {
      blk.push_back((int32_t)s);
      blk.push_back((int32_t)r0);
    }
  }
  const auto dev = x.device();
  auto d_off = to_dev_i32(off, dev), d_grp = to_dev_i32(grp, dev), d_blk = to_dev_i32(blk, dev);
  const int nb = (int)(blk.size() / 2);
  auto stream = at::cuda::getCurrentCUDAStream();
#define ART_LR_ROWS(RV)                                                                                          \
  lowrank_rows_kernel<RV><<<nb, 128, 0, stream>>>(                                                               \
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),                                         \
      src.has_value() ? src->data_ptr<int64_t>() : nullptr, scale.has_value() ? scale->data_ptr<float>() : nullptr, \
      d_off.data_ptr<int>(), d_grp.data_ptr<int>(), reinterpret_cast<const int2*>(d_blk.data_ptr<int>()),         \
      reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), w_gs, w_rs, w_ks, (int)K,                            \
      reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), y.stride(0))
  switch (R) {
    case 8: ART_LR_ROWS(8); break;
    case 16: ART_LR_ROWS(16); break;
    case 24: ART_LR_ROWS(24); break;
    case 32: ART_LR_ROWS(32); break;
    case 48: ART_LR_ROWS(48); break;
    case 64: ART_LR_ROWS(64); break;
    default: ART_LR_ROWS(96); break;
  }
#undef ART_LR_ROWS
  ART_CUDA_CHECK(cudaGetLastError());
  return y;
}

// G_g(r, c) += alpha * sum_{n in segment} P[n, r] * Q[n, c] for c < C, r < R;
// G fp32 addressed as g_gs * g + g_rs * r + g_cs * c.
void lowrank_wgrad(torch::Tensor p, torch::Tensor q, std::vector<int64_t> seg_off, std::vector<int64_t> seg_group,
                   torch::Tensor g, int64_t R, int64_t C, int64_t g_gs, int64_t g_rs, int64_t g_cs, double alpha) {
  TORCH_CHECK(p.is_cuda() && q.is_cuda() && g.is_cuda() && g.scalar_type() == at::kFloat);
  TORCH_CHECK(p.scalar_type() == at::kBFloat16 && q.scalar_type() == at::kBFloat16 && p.stride(1) == 1 && q.stride(1) == 1);
  TORCH_CHECK(p.stride(0) % 8 == 0 && q.stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(p.data_ptr()) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(q.data_ptr()) & 15) == 0,
              "rows 16-byte aligned");
  TORCH_CHECK(R == 8 || R == 16 || R == 24 || R == 32 || R == 48 || R == 64 || R == 96 || R == 128,
              "rank width 8/16/24/32/48/64/96/128");
  TORCH_CHECK(C % 8 == 0 && C <= q.size(1) && R <= p.size(1));
  const int64_t S = (int64_t)seg_group.size();
  TORCH_CHECK((int64_t)seg_off.size() == S + 1 && seg_off[0] == 0);
  const int64_t N = seg_off[S];
  TORCH_CHECK(p.size(0) >= N && q.size(0) >= N);
  if (N == 0 || C == 0) return;
  const int64_t ncol = (C + 127) / 128;
  // split long segments over several CTAs so the grid fills the GPU twice
  int64_t maxlen = 0;
  for (int64_t s = 0; s < S; ++s) maxlen = std::max<int64_t>(maxlen, seg_off[s + 1] - seg_off[s]);
  int64_t base_ctas = S * ncol;
  int splits = 1;
  while (base_ctas * splits < 2 * 148 && splits * 64 < maxlen) splits *= 2;
  std::vector<int32_t> off(S + 1), grp(S), blk;
  for (int64_t s = 0; s <= S; ++s) off[s] = (int32_t)seg_off[s];
  for (int64_t s = 0; s < S; ++s) {
    grp[s] = (int32_t)seg_group[s];
    if (seg_off[s + 1] == seg_off[s]) continue;
    for (int k = 0; k < splits; ++k) {
      blk.push_back((int32_t)s);
      blk.push_back(k);
    }
  }
  if (blk.empty()) return;
  const auto dev = p.device();
  auto d_off = to_dev_i32(off, dev), d_grp = to_dev_i32(grp, dev), d_blk = to_dev_i32(blk, dev);
  dim3 grid((unsigned)(blk.size() / 2), (unsigned)ncol);
  auto stream = at::cuda::getCurrentCUDAStream();
#define ART_LR_WG(RV)                                                                                            \
  lowrank_wgrad_kernel<RV><<<grid, 128, 0, stream>>>(                                                            \
      reinterpret_cast<const __nv_bfloat16*>(p.data_ptr()), p.stride(0),                                         \
      reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), q.stride(0), d_off.data_ptr<int>(),                  \
      d_grp.data_ptr<int>(), reinterpret_cast<const int2*>(d_blk.data_ptr<int>()), splits, (int)C,              \
      g.data_ptr<float>(), g_gs, g_rs, g_cs, (float)alpha)
  switch (R) {
    case 8: ART_LR_WG(8); break;
    case 16: ART_LR_WG(16); break;
    case 24: ART_LR_WG(24); break;
    case 32: ART_LR_WG(32); break;
    case 48: ART_LR_WG(48); break;
    case 64: ART_LR_WG(64); break;
    case 96: ART_LR_WG(96); break;
    default: ART_LR_WG(128); break;
  }
#undef ART_LR_WG
  ART_CUDA_CHECK(cudaGetLastError());
}

}  // namespace art
