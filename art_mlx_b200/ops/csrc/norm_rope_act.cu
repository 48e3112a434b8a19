// RMSNorm (+ fused residual add), qk-RMSNorm + RoPE on packed positions, and
// SwiGLU, forward and backward.  All memory-bound: one pass over the data,
// 16-byte vector accesses, fp32 math, bf16 storage.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "common.cuh"

namespace art {

// ----------------------------------------------------------------------------
// RMSNorm.  y = x_sum * rstd * w, x_sum = x (+ residual).  One CTA per row.
// The base-model norm weights are frozen, so the backward returns dx only.
// ----------------------------------------------------------------------------
template <int VEC>
__global__ void rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x,
                                   const __nv_bfloat16* __restrict__ res,
                                   const __nv_bfloat16* __restrict__ w,
                                   __nv_bfloat16* __restrict__ y,
                                   __nv_bfloat16* __restrict__ xsum,
                                   float* __restrict__ rstd, int H, float eps) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * H;
  const __nv_bfloat16* rr = res ? res + row * H : nullptr;
  float acc = 0.f;
  // pass 1: sum of squares (values kept in registers when they fit)
  constexpr int MAXV = 8;  // up to 8 vectors of 8 elements per thread (H <= 8*8*blockDim)
  float vals[MAXV][VEC];
  int nv = 0;
  for (int base = threadIdx.x * VEC; base < H; base += blockDim.x * VEC, ++nv) {
    uint4 xv = *reinterpret_cast<const uint4*>(xr + base);
    const __nv_bfloat16* xe = reinterpret_cast<const __nv_bfloat16*>(&xv);
    uint4 rv;
    const __nv_bfloat16* re = reinterpret_cast<const __nv_bfloat16*>(&rv);
    if (rr) rv = *reinterpret_cast<const uint4*>(rr + base);
#pragma unroll
    for (int k = 0; k < VEC; ++k) {
      float v = bf2f(xe[k]);
      if (rr) v = bf2f(f2bf(v + bf2f(re[k])));  // residual stream is stored in bf16
      vals[nv][k] = v;
      acc += v * v;
    }
  }
  float ss = block_sum(acc, red);
  float r = rsqrtf(ss / H + eps);
  if (threadIdx.x == 0) rstd[row] = r;
  nv = 0;
  for (int base = threadIdx.x * VEC; base < H; base += blockDim.x * VEC, ++nv) {
    uint4 wv = *reinterpret_cast<const uint4*>(w + base);
    const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv);
    uint4 out, sumv;
    __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&out);
    __nv_bfloat16* se = reinterpret_cast<__nv_bfloat16*>(&sumv);
#pragma unroll
    for (int k = 0; k < VEC; ++k) {
      // HF order: normalise in fp32, cast to bf16, then scale by the weight
      float n = bf2f(f2bf(vals[nv][k] * r));
      oe[k] = f2bf(n * bf2f(we[k]));
      se[k] = f2bf(vals[nv][k]);
    }
    *reinterpret_cast<uint4*>(y + row * H + base) = out;
    if (xsum) *reinterpret_cast<uint4*>(xsum + row * H + base) = sumv;
  }
}

// dx = rstd * (w*dy - xhat * mean(w*dy*xhat)) (+ dres)
template <int VEC>
__global__ void rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy,
                                   const __nv_bfloat16* __restrict__ xs,
                                   const __nv_bfloat16* __restrict__ w,
                                   const float* __restrict__ rstd,
                                   const __nv_bfloat16* __restrict__ dres,
                                   __nv_bfloat16* __restrict__ dx, int H) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const float r = rstd[row];
  constexpr int MAXV = 8;
  float g[MAXV][VEC], xh[MAXV][VEC];
  float acc = 0.f;
  int nv = 0;
  for (int base = threadIdx.x * VEC; base < H; base += blockDim.x * VEC, ++nv) {
    uint4 dv = *reinterpret_cast<const uint4*>(dy + row * H + base);
    uint4 xv = *reinterpret_cast<const uint4*>(xs + row * H + base);
    uint4 wv = *reinterpret_cast<const uint4*>(w + base);
    const __nv_bfloat16* de = reinterpret_cast<const __nv_bfloat16*>(&dv);
    const __nv_bfloat16* xe = reinterpret_cast<const __nv_bfloat16*>(&xv);
    const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv);
#pragma unroll
    for (int k = 0; k < VEC; ++k) {
      g[nv][k] = bf2f(de[k]) * bf2f(we[k]);
      xh[nv][k] = bf2f(xe[k]) * r;
      acc += g[nv][k] * xh[nv][k];
    }
  }
  const float mean = block_sum(acc, red) / H;
  nv = 0;
  for (int base = threadIdx.x * VEC; base < H; base += blockDim.x * VEC, ++nv) {
    uint4 out;
    __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&out);
    uint4 rv;
    const __nv_bfloat16* re = reinterpret_cast<const __nv_bfloat16*>(&rv);
    if (dres) rv = *reinterpret_cast<const uint4*>(dres + row * H + base);
#pragma unroll
    for (int k = 0; k < VEC; ++k) {
      float v = r * (g[nv][k] - xh[nv][k] * mean);
      if (dres) v += bf2f(re[k]);
      oe[k] = f2bf(v);
    }
    *reinterpret_cast<uint4*>(dx + row * H + base) = out;
  }
}

// Warp-per-row variants (hidden size = NV * 256): a warp owns one row and
// each lane NV 16-byte vectors of it (vector v*32 + lane, so a warp's loads are
// contiguous 512-byte runs), kept in registers as raw bf16 between the two
// passes (the backward re-reads its row through L2 in the second pass); the
// row reductions are warp shuffles, so there is no block barrier
// and a CTA of NORM_WARPS rows retires as soon as its warps do.  Same
// per-element arithmetic as the kernels above.
constexpr int NORM_WARPS = 4;

template <int NV>
__global__ void __launch_bounds__(NORM_WARPS * 32) rmsnorm_fwd_warp_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ res, const __nv_bfloat16* __restrict__ w,
    __nv_bfloat16* __restrict__ y, __nv_bfloat16* __restrict__ xsum, float* __restrict__ rstd, int64_t T, int H,
    float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * NORM_WARPS + (threadIdx.x >> 5);
  if (row >= T) return;  // warp-uniform
  const __nv_bfloat16* xr = x + row * H;
  uint4 xv[NV];
#pragma unroll
  for (int v = 0; v < NV; ++v) xv[v] = *reinterpret_cast<const uint4*>(xr + (v * 32 + lane) * 8);
  float acc = 0.f;
  if (res) {
    const __nv_bfloat16* rr = res + row * H;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const uint4 rv = *reinterpret_cast<const uint4*>(rr + (v * 32 + lane) * 8);
      __nv_bfloat16* xe = reinterpret_cast<__nv_bfloat16*>(&xv[v]);
      const __nv_bfloat16* re = reinterpret_cast<const __nv_bfloat16*>(&rv);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        xe[k] = f2bf(bf2f(xe[k]) + bf2f(re[k]));  // residual stream is stored in bf16
        const float a = bf2f(xe[k]);
        acc += a * a;
      }
    }
  } else {
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const __nv_bfloat16* xe = reinterpret_cast<const __nv_bfloat16*>(&xv[v]);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float a = bf2f(xe[k]);
        acc += a * a;
      }
    }
  }
  const float r = rsqrtf(warp_sum(acc) / H + eps);
  if (lane == 0) rstd[row] = r;
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int64_t off = row * H + (v * 32 + lane) * 8;
    const uint4 wv = *reinterpret_cast<const uint4*>(w + (v * 32 + lane) * 8);
    const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv);
    const __nv_bfloat16* xe = reinterpret_cast<const __nv_bfloat16*>(&xv[v]);
    uint4 out;
    __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&out);
#pragma unroll
    for (int k = 0; k < 8; ++k) oe[k] = f2bf(bf2f(f2bf(bf2f(xe[k]) * r)) * bf2f(we[k]));
    *reinterpret_cast<uint4*>(y + off) = out;
    if (xsum) *reinterpret_cast<uint4*>(xsum + off) = xv[v];
  }
}

// 16-byte load that stays a separate load (L2, not L1): the backward's second
// pass re-reads the row instead of keeping it in registers.
__device__ __forceinline__ uint4 ld_cg16(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

template <int NV>
__global__ void __launch_bounds__(NORM_WARPS * 32) rmsnorm_bwd_warp_kernel(
    const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ xs, const __nv_bfloat16* __restrict__ w,
    const float* __restrict__ rstd, const __nv_bfloat16* __restrict__ dres, __nv_bfloat16* __restrict__ dx, int64_t T,
    int H) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * NORM_WARPS + (threadIdx.x >> 5);
  if (row >= T) return;  // warp-uniform
  const float r = rstd[row];
  // pass 1: mean(w*dy*xhat); the row's dy and x come from HBM here
  float acc = 0.f;
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int64_t off = row * H + (v * 32 + lane) * 8;
    const uint4 dv = *reinterpret_cast<const uint4*>(dy + off);
    const uint4 xv = *reinterpret_cast<const uint4*>(xs + off);
    const uint4 wv = *reinterpret_cast<const uint4*>(w + (v * 32 + lane) * 8);
    const __nv_bfloat16* de = reinterpret_cast<const __nv_bfloat16*>(&dv);
    const __nv_bfloat16* xe = reinterpret_cast<const __nv_bfloat16*>(&xv);
    const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv);
#pragma unroll
    for (int k = 0; k < 8; ++k) acc += (bf2f(de[k]) * bf2f(we[k])) * (bf2f(xe[k]) * r);
  }
  const float mean = warp_sum(acc) / H;
  // pass 2: dx, re-reading dy and x from L2
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int64_t off = row * H + (v * 32 + lane) * 8;
    const uint4 dv = ld_cg16(dy + off);
    const uint4 xv = ld_cg16(xs + off);
    const uint4 wv = *reinterpret_cast<const uint4*>(w + (v * 32 + lane) * 8);
    const __nv_bfloat16* de = reinterpret_cast<const __nv_bfloat16*>(&dv);
    const __nv_bfloat16* xe = reinterpret_cast<const __nv_bfloat16*>(&xv);
    const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv);
    uint4 rv;
    const __nv_bfloat16* re = reinterpret_cast<const __nv_bfloat16*>(&rv);
    if (dres) rv = *reinterpret_cast<const uint4*>(dres + off);
    uint4 out;
    __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&out);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float val = r * (bf2f(de[k]) * bf2f(we[k]) - (bf2f(xe[k]) * r) * mean);
      if (dres) val += bf2f(re[k]);
      oe[k] = f2bf(val);
    }
    *reinterpret_cast<uint4*>(dx + off) = out;
  }
}

// Hidden sizes with a warp-per-row instantiation (H = NV * 256).
#define ART_NORM_NV(X) X(1) X(2) X(4) X(6) X(8) X(10) X(12) X(14) X(16) X(20) X(24)
#define ART_NORM_NV_BWD(X) ART_NORM_NV(X)

static bool norm_warp_ok(int H, bool bwd) {
  if (H % 256 != 0) return false;
  switch (H / 256) {
#define ART_CASE(n) case n:
    ART_NORM_NV_BWD(ART_CASE)
#undef ART_CASE
    return true;
    default:
      return false;
  }
}

static int norm_threads(int H) {
  int t = (H / 8 + 7) / 8;  // 8 vectors of 8 per thread at most
  t = ((t + 31) / 32) * 32;
  if (t < 64) t = 64;
  if (t > 1024) t = 1024;
  return t;
}

std::vector<torch::Tensor> rmsnorm_fwd(torch::Tensor x, c10::optional<torch::Tensor> res,
                                       torch::Tensor w, double eps, bool legacy) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous());
  const int H = x.size(-1);
  TORCH_CHECK(H % 8 == 0 && H <= 8 * 8 * 1024, "rmsnorm: hidden size must be a multiple of 8");
  const int64_t T = x.numel() / H;
  auto y = torch::empty_like(x);
  auto rstd = torch::empty({T}, x.options().dtype(at::kFloat));
  torch::Tensor xs;
  const __nv_bfloat16* rp = nullptr;
  __nv_bfloat16* xsp = nullptr;
  if (res.has_value()) {
    TORCH_CHECK(res->is_contiguous() && res->sizes() == x.sizes());
    xs = torch::empty_like(x);
    rp = reinterpret_cast<const __nv_bfloat16*>(res->data_ptr());
    xsp = reinterpret_cast<__nv_bfloat16*>(xs.data_ptr());
  } else {
    xs = x;
  }
  auto st = at::cuda::getCurrentCUDAStream();
  const auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  const auto* wp = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  auto* yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  if (T > 0 && !legacy && norm_warp_ok(H, false)) {
    const unsigned grid = (unsigned)((T + NORM_WARPS - 1) / NORM_WARPS);
    switch (H / 256) {
#define ART_CASE(n)                                                                                          \
  case n:                                                                                                    \
    rmsnorm_fwd_warp_kernel<n><<<grid, NORM_WARPS * 32, 0, st>>>(xp, rp, wp, yp, xsp, rstd.data_ptr<float>(), T, \
                                                                 H, (float)eps);                             \
    break;
      ART_NORM_NV(ART_CASE)
#undef ART_CASE
    }
  } else if (T > 0) {
    rmsnorm_fwd_kernel<8><<<T, norm_threads(H), 0, st>>>(xp, rp, wp, yp, xsp, rstd.data_ptr<float>(), H, (float)eps);
  }
  ART_CUDA_CHECK(cudaGetLastError());
  return {y, xs, rstd};
}

torch::Tensor rmsnorm_bwd(torch::Tensor dy, torch::Tensor xs, torch::Tensor w, torch::Tensor rstd,
                          c10::optional<torch::Tensor> dres, bool legacy) {
  TORCH_CHECK(dy.is_contiguous() && xs.is_contiguous());
  const int H = dy.size(-1);
  const int64_t T = dy.numel() / H;
  auto dx = torch::empty_like(dy);
  const __nv_bfloat16* dr = nullptr;
  if (dres.has_value()) {
    TORCH_CHECK(dres->is_contiguous());
    dr = reinterpret_cast<const __nv_bfloat16*>(dres->data_ptr());
  }
  auto st = at::cuda::getCurrentCUDAStream();
  const auto* dyp = reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr());
  const auto* xsp = reinterpret_cast<const __nv_bfloat16*>(xs.data_ptr());
  const auto* wp = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  auto* dxp = reinterpret_cast<__nv_bfloat16*>(dx.data_ptr());
  if (T > 0 && !legacy && norm_warp_ok(H, true)) {
    const unsigned grid = (unsigned)((T + NORM_WARPS - 1) / NORM_WARPS);
    switch (H / 256) {
#define ART_CASE(n)                                                                                          \
  case n:                                                                                                    \
    rmsnorm_bwd_warp_kernel<n><<<grid, NORM_WARPS * 32, 0, st>>>(dyp, xsp, wp, rstd.data_ptr<float>(), dr, dxp, T, H); \
    break;
      ART_NORM_NV_BWD(ART_CASE)
#undef ART_CASE
    }
  } else if (T > 0) {
    rmsnorm_bwd_kernel<8><<<T, norm_threads(H), 0, st>>>(dyp, xsp, wp, rstd.data_ptr<float>(), dr, dxp, H);
  }
  ART_CUDA_CHECK(cudaGetLastError());
  return dx;
}

// ----------------------------------------------------------------------------
// qk-RMSNorm (optional) + RoPE (rotate-half convention) on packed positions.
// Input: raw projection output qkv [T, (nq + 2*nkv) * D] (row stride ld).
// Output: qk [T, (nq + nkv) * D] rotated q then k heads; rstd [T, nq + nkv].
// One warp per (token, head); D in {64, 128, 256}.
// ----------------------------------------------------------------------------
template <int D>
__global__ void rope_fwd_kernel(const __nv_bfloat16* __restrict__ qkv, int64_t ld,
                                const int* __restrict__ pos, const float* __restrict__ inv_freq,
                                const __nv_bfloat16* __restrict__ qn_w,
                                const __nv_bfloat16* __restrict__ kn_w,
                                __nv_bfloat16* __restrict__ out, float* __restrict__ rstd_out,
                                int64_t T, int nq, int nkv, float eps, const short* __restrict__ perm) {
  constexpr int PER = D / 32;  // elements per lane; lane owns pairs (i, i + D/2)
  // perm (optional): column of the head that internal element i is read from
  // (partial rotary: the rotated dims and their partners moved to the pair
  // layout, the rest paired with zero frequencies); out keeps internal order
#define ART_P(i) (perm ? (int)__ldg(perm + (i)) : (i))
  const int nh = nq + nkv;
  const int64_t gw = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x / 32);
  const int lane = threadIdx.x & 31;
  if (gw >= T * nh) return;
  const int64_t t = gw / nh;
  const int h = gw % nh;
  const bool is_q = h < nq;
  const __nv_bfloat16* src = qkv + t * ld + (int64_t)h * D;
  const __nv_bfloat16* nw = is_q ? qn_w : kn_w;
  // lane holds x[i] for i = lane*PER/2 .. and the rotation partner at +D/2
  float a[PER / 2], b[PER / 2];
#pragma unroll
  for (int k = 0; k < PER / 2; ++k) {
    a[k] = bf2f(src[ART_P(lane * (PER / 2) + k)]);
    b[k] = bf2f(src[ART_P(D / 2 + lane * (PER / 2) + k)]);
  }
  float r = 1.f;
  if (nw) {
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < PER / 2; ++k) ss += a[k] * a[k] + b[k] * b[k];
    ss = warp_sum(ss);
    r = rsqrtf(ss / D + eps);
#pragma unroll
    for (int k = 0; k < PER / 2; ++k) {
      const int i = lane * (PER / 2) + k;
      a[k] = bf2f(f2bf(a[k] * r)) * bf2f(nw[ART_P(i)]);
      b[k] = bf2f(f2bf(b[k] * r)) * bf2f(nw[ART_P(i + D / 2)]);
      a[k] = bf2f(f2bf(a[k]));
      b[k] = bf2f(f2bf(b[k]));
    }
  }
  if (rstd_out && lane == 0) rstd_out[t * nh + h] = r;
  const float p = (float)pos[t];
  __nv_bfloat16* dst = out + t * (int64_t)nh * D + (int64_t)h * D;
#pragma unroll
  for (int k = 0; k < PER / 2; ++k) {
    const int i = lane * (PER / 2) + k;
    float s, c;
    sincosf(p * inv_freq[i], &s, &c);
    dst[i] = f2bf(a[k] * c - b[k] * s);
    dst[i + D / 2] = f2bf(b[k] * c + a[k] * s);
  }
}

// Backward: dqk [T, nh*D] (bf16) -> writes dq, dk into dqkv [T, ld] columns of q and k.
// Needs the raw (pre-norm) input to redo the norm when qk-norm is on.
template <int D>
__device__ __forceinline__ float grad_f(float x) { return x; }
__device__ __forceinline__ float grad_f(__nv_bfloat16 x) { return bf2f(x); }

// Gradients of q and k arrive as G (bf16, or the fp32 accumulators of the
// attention backward) at row strides ldq / ldk and head stride hs; with
// nv > 0 the value gradient (fp32 [T, nv, hs]) is converted into its slice of
// dqkv by the same launch (warps past the q and k heads).
template <int D, typename G>
__global__ void rope_bwd_kernel(const G* __restrict__ dq, const G* __restrict__ dk, int64_t ldq, int64_t ldk,
                                int hs, const float* __restrict__ dv, int nv,
                                const __nv_bfloat16* __restrict__ qkv, int64_t ld,
                                const int* __restrict__ pos, const float* __restrict__ inv_freq,
                                const __nv_bfloat16* __restrict__ qn_w,
                                const __nv_bfloat16* __restrict__ kn_w,
                                const float* __restrict__ rstd, __nv_bfloat16* __restrict__ dqkv,
                                int64_t T, int nq, int nkv, const short* __restrict__ perm) {
  constexpr int PER = D / 32;
  const int nh = nq + nkv;
  const int nwarp = nh + nv;
  const int64_t gw = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x / 32);
  const int lane = threadIdx.x & 31;
  if (gw >= T * nwarp) return;
  const int64_t t = gw / nwarp;
  const int h = gw % nwarp;
  if (h >= nh) {  // value gradient: fp32 -> bf16 into its slice
    const float* src = dv + (t * nv + (h - nh)) * (int64_t)hs;
    __nv_bfloat16* dst = dqkv + t * ld + (int64_t)h * D;
#pragma unroll
    for (int k = 0; k < PER; ++k) dst[lane + 32 * k] = f2bf(src[lane + 32 * k]);
    return;
  }
  const bool is_q = h < nq;
  const G* g = is_q ? dq + t * ldq + (int64_t)h * hs : dk + t * ldk + (int64_t)(h - nq) * hs;
  const float p = (float)pos[t];
  float ga[PER / 2], gb[PER / 2];
#pragma unroll
  for (int k = 0; k < PER / 2; ++k) {
    const int i = lane * (PER / 2) + k;
    float s, c;
    sincosf(p * inv_freq[i], &s, &c);
    const float u = grad_f(g[i]), v = grad_f(g[i + D / 2]);
    // transpose of the rotation
    ga[k] = u * c + v * s;
    gb[k] = v * c - u * s;
  }
  const __nv_bfloat16* nw = is_q ? qn_w : kn_w;
  __nv_bfloat16* dst = dqkv + t * ld + (int64_t)h * D;
  if (nw) {
    const __nv_bfloat16* src = qkv + t * ld + (int64_t)h * D;
    const float r = rstd[t * nh + h];
    float xa[PER / 2], xb[PER / 2];
    float dot = 0.f;
#pragma unroll
    for (int k = 0; k < PER / 2; ++k) {
      const int i = lane * (PER / 2) + k;
      xa[k] = bf2f(src[ART_P(i)]) * r;
      xb[k] = bf2f(src[ART_P(i + D / 2)]) * r;
      ga[k] *= bf2f(nw[ART_P(i)]);
      gb[k] *= bf2f(nw[ART_P(i + D / 2)]);
      dot += ga[k] * xa[k] + gb[k] * xb[k];
    }
    const float mean = warp_sum(dot) / D;
#pragma unroll
    for (int k = 0; k < PER / 2; ++k) {
      const int i = lane * (PER / 2) + k;
      dst[ART_P(i)] = f2bf(r * (ga[k] - xa[k] * mean));
      dst[ART_P(i + D / 2)] = f2bf(r * (gb[k] - xb[k] * mean));
    }
  } else {
#pragma unroll
    for (int k = 0; k < PER / 2; ++k) {
      const int i = lane * (PER / 2) + k;
      dst[ART_P(i)] = f2bf(ga[k]);
      dst[ART_P(i + D / 2)] = f2bf(gb[k]);
    }
  }
}
#undef ART_P

#define ART_DISPATCH_HEAD_DIM(D, ...)                       \
  [&] {                                                     \
    if (D == 64) {                                          \
      constexpr int kD = 64;                                \
      return __VA_ARGS__();                                 \
    } else if (D == 128) {                                  \
      constexpr int kD = 128;                               \
      return __VA_ARGS__();                                 \
    } else if (D == 256) {                                  \
      constexpr int kD = 256;                               \
      return __VA_ARGS__();                                 \
    }                                                       \
    TORCH_CHECK(false, "unsupported head_dim ", D);         \
  }()

std::vector<torch::Tensor> rope_fwd(torch::Tensor qkv, torch::Tensor pos, torch::Tensor inv_freq,
                                    int64_t nq, int64_t nkv, int64_t D,
                                    c10::optional<torch::Tensor> qn_w,
                                    c10::optional<torch::Tensor> kn_w, double eps,
                                    c10::optional<torch::Tensor> perm) {
  TORCH_CHECK(qkv.stride(-1) == 1 && pos.scalar_type() == at::kInt && pos.is_contiguous());
  if (perm.has_value())
    TORCH_CHECK(perm->is_cuda() && perm->scalar_type() == at::kShort && perm->numel() == D && perm->is_contiguous(),
                "perm: int16 [head_dim]");
  const short* pp = perm.has_value() ? perm->data_ptr<short>() : nullptr;
  const int64_t T = qkv.size(0);
  const int64_t ld = qkv.stride(0);
  const int nh = nq + nkv;
  auto out = torch::empty({T, nh * D}, qkv.options());
  const bool norm = qn_w.has_value();
  auto rstd = norm ? torch::empty({T, nh}, qkv.options().dtype(at::kFloat)) : torch::Tensor();
  const int64_t warps = T * nh;
  const int threads = 256;
  const int64_t blocks = (warps + threads / 32 - 1) / (threads / 32);
  if (warps > 0)
    ART_DISPATCH_HEAD_DIM(D, [&] {
      rope_fwd_kernel<kD><<<blocks, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
          reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), ld, pos.data_ptr<int>(),
          inv_freq.data_ptr<float>(),
          norm ? reinterpret_cast<const __nv_bfloat16*>(qn_w->data_ptr()) : nullptr,
          norm ? reinterpret_cast<const __nv_bfloat16*>(kn_w->data_ptr()) : nullptr,
          reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), norm ? rstd.data_ptr<float>() : nullptr,
          T, (int)nq, (int)nkv, (float)eps, pp);
    });
  ART_CUDA_CHECK(cudaGetLastError());
  return {out, rstd};
}

void rope_bwd(torch::Tensor dqk, torch::Tensor qkv, torch::Tensor pos, torch::Tensor inv_freq,
              int64_t nq, int64_t nkv, int64_t D, c10::optional<torch::Tensor> qn_w,
              c10::optional<torch::Tensor> kn_w, c10::optional<torch::Tensor> rstd,
              torch::Tensor dqkv, c10::optional<torch::Tensor> perm) {
  TORCH_CHECK(dqk.is_contiguous() && dqkv.stride(-1) == 1 && dqkv.stride(0) == qkv.stride(0));
  if (perm.has_value())
    TORCH_CHECK(perm->is_cuda() && perm->scalar_type() == at::kShort && perm->numel() == D && perm->is_contiguous(),
                "perm: int16 [head_dim]");
  const short* pp = perm.has_value() ? perm->data_ptr<short>() : nullptr;
  const int64_t T = dqk.size(0);
  const int nh = nq + nkv;
  const int64_t warps = T * nh;
  const int threads = 256;
  const int64_t blocks = (warps + threads / 32 - 1) / (threads / 32);
  const bool norm = qn_w.has_value();
  const __nv_bfloat16* g = reinterpret_cast<const __nv_bfloat16*>(dqk.data_ptr());
  if (warps > 0)
    ART_DISPATCH_HEAD_DIM(D, [&] {
      rope_bwd_kernel<kD, __nv_bfloat16><<<blocks, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
          g, g + nq * D, (int64_t)nh * D, (int64_t)nh * D, (int)D, nullptr, 0,
          reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), qkv.stride(0),
          pos.data_ptr<int>(), inv_freq.data_ptr<float>(),
          norm ? reinterpret_cast<const __nv_bfloat16*>(qn_w->data_ptr()) : nullptr,
          norm ? reinterpret_cast<const __nv_bfloat16*>(kn_w->data_ptr()) : nullptr,
          norm ? rstd->data_ptr<float>() : nullptr,
          reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()), T, (int)nq, (int)nkv, pp);
    });
  ART_CUDA_CHECK(cudaGetLastError());
}

// The attention backward's fp32 accumulators dq [T, nq, hs], dk / dv
// [T, nkv, hs] (hs >= D: narrow heads are padded) straight into dqkv: q and k
// through the RoPE / q-k-norm backward, v converted, one launch, no bf16
// intermediate.
void rope_bwd_f32(torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor qkv, torch::Tensor pos,
                  torch::Tensor inv_freq, int64_t nq, int64_t nkv, int64_t D, c10::optional<torch::Tensor> qn_w,
                  c10::optional<torch::Tensor> kn_w, c10::optional<torch::Tensor> rstd, torch::Tensor dqkv,
                  c10::optional<torch::Tensor> perm) {
  for (auto* t : {&dq, &dk, &dv})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous() && t->dim() == 3 &&
                    t->size(2) >= D && t->size(0) == qkv.size(0),
                "fp32 contiguous [T, heads, >= head_dim]");
  TORCH_CHECK(dq.size(1) == nq && dk.size(1) == nkv && dv.size(1) == nkv && dk.size(2) == dq.size(2) &&
                  dv.size(2) == dq.size(2),
              "dq [T, nq, hs], dk / dv [T, nkv, hs]");
  TORCH_CHECK(dqkv.stride(-1) == 1 && dqkv.stride(0) == qkv.stride(0) && dqkv.size(1) >= (nq + 2 * nkv) * D);
  if (perm.has_value())
    TORCH_CHECK(perm->is_cuda() && perm->scalar_type() == at::kShort && perm->numel() == D && perm->is_contiguous(),
                "perm: int16 [head_dim]");
  const short* pp = perm.has_value() ? perm->data_ptr<short>() : nullptr;
  const int64_t T = qkv.size(0);
  const int hs = (int)dq.size(2);
  const int64_t warps = T * (nq + 2 * nkv);
  const int threads = 256;
  const int64_t blocks = (warps + threads / 32 - 1) / (threads / 32);
  const bool norm = qn_w.has_value();
  if (warps > 0)
    ART_DISPATCH_HEAD_DIM(D, [&] {
      rope_bwd_kernel<kD, float><<<blocks, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
          dq.data_ptr<float>(), dk.data_ptr<float>(), (int64_t)nq * hs, (int64_t)nkv * hs, hs, dv.data_ptr<float>(),
          (int)nkv, reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), qkv.stride(0), pos.data_ptr<int>(),
          inv_freq.data_ptr<float>(), norm ? reinterpret_cast<const __nv_bfloat16*>(qn_w->data_ptr()) : nullptr,
          norm ? reinterpret_cast<const __nv_bfloat16*>(kn_w->data_ptr()) : nullptr, norm ? rstd->data_ptr<float>() : nullptr,
          reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()), T, (int)nq, (int)nkv, pp);
    });
  ART_CUDA_CHECK(cudaGetLastError());
}

// ----------------------------------------------------------------------------
// SwiGLU: gu = [gate | up] per row (width 2F) -> a = silu(gate) * up.
// ----------------------------------------------------------------------------
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ a,
                                  int64_t T, int F) {
  const int64_t nvec = T * (F / 8);
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nvec;
       v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = v / (F / 8);
    const int c = (v % (F / 8)) * 8;
    uint4 gv = *reinterpret_cast<const uint4*>(gu + t * 2 * F + c);
    uint4 uv = *reinterpret_cast<const uint4*>(gu + t * 2 * F + F + c);
    const __nv_bfloat16* ge = reinterpret_cast<const __nv_bfloat16*>(&gv);
    const __nv_bfloat16* ue = reinterpret_cast<const __nv_bfloat16*>(&uv);
    uint4 ov;
    __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&ov);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float g = bf2f(ge[k]);
      const float s = g / (1.f + __expf(-g));
      oe[k] = f2bf(bf2f(f2bf(s)) * bf2f(ue[k]));
    }
    *reinterpret_cast<uint4*>(a + t * F + c) = ov;
  }
}

__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ da,
                                  const __nv_bfloat16* __restrict__ gu,
                                  __nv_bfloat16* __restrict__ dgu, int64_t T, int F) {
  const int64_t nvec = T * (F / 8);
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nvec;
       v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = v / (F / 8);
    const int c = (v % (F / 8)) * 8;
    uint4 dv = *reinterpret_cast<const uint4*>(da + t * F + c);
    uint4 gv = *reinterpret_cast<const uint4*>(gu + t * 2 * F + c);
    uint4 uv = *reinterpret_cast<const uint4*>(gu + t * 2 * F + F + c);
    const __nv_bfloat16* de = reinterpret_cast<const __nv_bfloat16*>(&dv);
    const __nv_bfloat16* ge = reinterpret_cast<const __nv_bfloat16*>(&gv);
    const __nv_bfloat16* ue = reinterpret_cast<const __nv_bfloat16*>(&uv);
    uint4 dg, du;
    __nv_bfloat16* dge = reinterpret_cast<__nv_bfloat16*>(&dg);
    __nv_bfloat16* due = reinterpret_cast<__nv_bfloat16*>(&du);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float g = bf2f(ge[k]), u = bf2f(ue[k]), d = bf2f(de[k]);
      const float sg = 1.f / (1.f + __expf(-g));
      const float s = g * sg;
      due[k] = f2bf(d * s);
      dge[k] = f2bf(d * u * sg * (1.f + g * (1.f - sg)));
    }
    *reinterpret_cast<uint4*>(dgu + t * 2 * F + c) = dg;
    *reinterpret_cast<uint4*>(dgu + t * 2 * F + F + c) = du;
  }
}

static int64_t ew_blocks(int64_t n) {
  int64_t b = (n + 255) / 256;
  const int64_t cap = 148 * 16;
  return b < 1 ? 1 : (b > cap ? cap : b);
}

torch::Tensor swiglu_fwd(torch::Tensor gu) {
  TORCH_CHECK(gu.is_contiguous() && gu.size(-1) % 16 == 0);
  const int F = gu.size(-1) / 2;
  const int64_t T = gu.numel() / (2 * F);
  auto sizes = gu.sizes().vec();
  sizes.back() = F;
  auto a = torch::empty(sizes, gu.options());
  if (T > 0)
    swiglu_fwd_kernel<<<ew_blocks(T * F / 8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()),
        reinterpret_cast<__nv_bfloat16*>(a.data_ptr()), T, F);
  ART_CUDA_CHECK(cudaGetLastError());
  return a;
}

torch::Tensor swiglu_bwd(torch::Tensor da, torch::Tensor gu) {
  TORCH_CHECK(da.is_contiguous() && gu.is_contiguous());
  const int F = gu.size(-1) / 2;
  const int64_t T = gu.numel() / (2 * F);
  auto dgu = torch::empty_like(gu);
  if (T > 0)
    swiglu_bwd_kernel<<<ew_blocks(T * F / 8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(da.data_ptr()),
        reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()),
        reinterpret_cast<__nv_bfloat16*>(dgu.data_ptr()), T, F);
  ART_CUDA_CHECK(cudaGetLastError());
  return dgu;
}

// Clamped GLU of the GPT-OSS experts over a [gate | up] row:
//   g' = min(g, limit), u' = clamp(u, -limit, limit)
//   a  = (u' + 1) * g' * sigmoid(alpha * g')
// Backward: d up = da * g' sigmoid(alpha g') where |u| <= limit (else 0);
//           d gate = da * (u' + 1) * (s + alpha g' s (1 - s)) where g <= limit.
__global__ void glu_clamp_fwd_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ a, int64_t T,
                                     int F, float alpha, float limit) {
  const int64_t nvec = T * (F / 8);
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = v / (F / 8);
    const int c = (v % (F / 8)) * 8;
    uint4 gv = *reinterpret_cast<const uint4*>(gu + t * 2 * F + c);
    uint4 uv = *reinterpret_cast<const uint4*>(gu + t * 2 * F + F + c);
    const __nv_bfloat16* ge = reinterpret_cast<const __nv_bfloat16*>(&gv);
    const __nv_bfloat16* ue = reinterpret_cast<const __nv_bfloat16*>(&uv);
    uint4 ov;
    __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&ov);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float g = fminf(bf2f(ge[k]), limit);
      const float u = fminf(fmaxf(bf2f(ue[k]), -limit), limit);
      const float sg = 1.f / (1.f + __expf(-alpha * g));
      oe[k] = f2bf((u + 1.f) * g * sg);
    }
    *reinterpret_cast<uint4*>(a + t * F + c) = ov;
  }
}

__global__ void glu_clamp_bwd_kernel(const __nv_bfloat16* __restrict__ da, const __nv_bfloat16* __restrict__ gu,
                                     __nv_bfloat16* __restrict__ dgu, int64_t T, int F, float alpha, float limit) {
  const int64_t nvec = T * (F / 8);
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = v / (F / 8);
    const int c = (v % (F / 8)) * 8;
    uint4 dv = *reinterpret_cast<const uint4*>(da + t * F + c);
    uint4 gv = *reinterpret_cast<const uint4*>(gu + t * 2 * F + c);
    uint4 uv = *reinterpret_cast<const uint4*>(gu + t * 2 * F + F + c);
    const __nv_bfloat16* de = reinterpret_cast<const __nv_bfloat16*>(&dv);
    const __nv_bfloat16* ge = reinterpret_cast<const __nv_bfloat16*>(&gv);
    const __nv_bfloat16* ue = reinterpret_cast<const __nv_bfloat16*>(&uv);
    uint4 dg, du;
    __nv_bfloat16* dge = reinterpret_cast<__nv_bfloat16*>(&dg);
    __nv_bfloat16* due = reinterpret_cast<__nv_bfloat16*>(&du);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float graw = bf2f(ge[k]), uraw = bf2f(ue[k]), d = bf2f(de[k]);
      const float g = fminf(graw, limit);
      const float u = fminf(fmaxf(uraw, -limit), limit);
      const float sg = 1.f / (1.f + __expf(-alpha * g));
      const float glu = g * sg;
      due[k] = f2bf((uraw >= -limit && uraw <= limit) ? d * glu : 0.f);
      dge[k] = f2bf(graw <= limit ? d * (u + 1.f) * (sg + alpha * g * sg * (1.f - sg)) : 0.f);
    }
    *reinterpret_cast<uint4*>(dgu + t * 2 * F + c) = dg;
    *reinterpret_cast<uint4*>(dgu + t * 2 * F + F + c) = du;
  }
}

torch::Tensor glu_clamp_fwd(torch::Tensor gu, double alpha, double limit) {
  TORCH_CHECK(gu.is_cuda() && gu.scalar_type() == at::kBFloat16 && gu.is_contiguous() && gu.size(-1) % 16 == 0);
  const int F = gu.size(-1) / 2;
  const int64_t T = gu.numel() / (2 * F);
  auto sizes = gu.sizes().vec();
  sizes.back() = F;
  auto a = torch::empty(sizes, gu.options());
  if (T > 0)
    glu_clamp_fwd_kernel<<<ew_blocks(T * F / 8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()), reinterpret_cast<__nv_bfloat16*>(a.data_ptr()), T, F,
        (float)alpha, (float)limit);
  ART_CUDA_CHECK(cudaGetLastError());
  return a;
}

torch::Tensor glu_clamp_bwd(torch::Tensor da, torch::Tensor gu, double alpha, double limit) {
  TORCH_CHECK(da.is_contiguous() && gu.is_contiguous() && gu.scalar_type() == at::kBFloat16);
  const int F = gu.size(-1) / 2;
  const int64_t T = gu.numel() / (2 * F);
  TORCH_CHECK(da.numel() == T * F, "da must be [T, F]");
  auto dgu = torch::empty_like(gu);
  if (T > 0)
    glu_clamp_bwd_kernel<<<ew_blocks(T * F / 8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(da.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()),
        reinterpret_cast<__nv_bfloat16*>(dgu.data_ptr()), T, F, (float)alpha, (float)limit);
  ART_CUDA_CHECK(cudaGetLastError());
  return dgu;
}

}  // namespace art
