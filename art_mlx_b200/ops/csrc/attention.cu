// Prefix-tree (shared-prompt) causal attention, forward and backward, GQA,
// head_dim 128, bf16 in / fp32 accumulate, natural-log LSE output.
//
// Mask: key j is visible to query i iff  j <= i < kend[j].  The packer emits
// prefix-tree segments in depth-first pre-order, so `kend[j]` (the end of the
// subtree of j's segment) expresses "full attention to every ancestor segment,
// causal inside the own segment" with one int per key.  Key tiles whose
// largest kend does not reach the query block are skipped without loading.
//
// This is the warp-level (mma.sync m16n8k16) implementation: flash-attention
// style online softmax in registers, K/V tiles double-buffered with cp.async
// into XOR-swizzled shared memory.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "common.cuh"
#include "art_noalloc.h"

namespace art {

constexpr float kLog2e = 1.4426950408889634f;

// ----------------------------------------------------------------------------
// Forward: CTA = 64 queries x one q head; 4 warps x 16 query rows; 64-key tiles.
// ----------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(128) attn_fwd_kernel(
    const __nv_bfloat16* __restrict__ q, int64_t ldq, const __nv_bfloat16* __restrict__ k,
    int64_t ldk, const __nv_bfloat16* __restrict__ v, int64_t ldv, const int* __restrict__ kend,
    const int* __restrict__ tile_kmax, __nv_bfloat16* __restrict__ o, int64_t ldo,
    float* __restrict__ lse, int Tq, int Tk, int q_off, int Hq, int Hkv, float scale_log2) {
  static_assert(D == 128, "head_dim 128");
  // queries are local rows [0, Tq) at global positions q_off + row; keys are
  // global rows [0, Tk) (Tq == Tk, q_off == 0 without context parallelism)
  constexpr int CH = D / 8;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  __nv_bfloat16* sK = sQ + 64 * D;
  __nv_bfloat16* sV = sK + 2 * 64 * D;

  const int q0 = blockIdx.x * 64;
  const int h = blockIdx.y;
  const int hk = h / (Hq / Hkv);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  for (int c = tid; c < 64 * CH; c += 128) {
    const int r = c / CH, ch = c % CH;
    const int t = q0 + r;
    const int tt = t < Tq ? t : Tq - 1;
    cp_async16(smem_u32(sQ + swz<D>(r, ch)), q + (int64_t)tt * ldq + h * D + ch * 8, t < Tq ? 16 : 0);
  }
  cp_async_commit();

  const int gq0 = q_off + q0;  // global position of the first query of the block
  const int q_last = min(gq0 + 63, q_off + Tq - 1);
  const int ntiles = min(q_last / 64 + 1, (Tk + 63) / 64);
  auto next_needed = [&](int t) {
    while (t < ntiles && __ldg(tile_kmax + t) <= gq0) ++t;
    return t;
  };
  auto load_kv = [&](int tile, int stage) {
    const int j0 = tile * 64;
    for (int c = tid; c < 64 * CH; c += 128) {
      const int r = c / CH, ch = c % CH;
      const int j = j0 + r;
      const int jj = j < Tk ? j : Tk - 1;
      const int nb = j < Tk ? 16 : 0;
      cp_async16(smem_u32(sK + stage * 64 * D + swz<D>(r, ch)), k + (int64_t)jj * ldk + hk * D + ch * 8, nb);
      cp_async16(smem_u32(sV + stage * 64 * D + swz<D>(r, ch)), v + (int64_t)jj * ldv + hk * D + ch * 8, nb);
    }
  };

  int tile = next_needed(0);
  if (tile < ntiles) load_kv(tile, 0);
  cp_async_commit();

  cp_async_wait<1>();
  __syncthreads();
  uint32_t qf[D / 16][4];
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk)
    ldsm_x4(qf[kk], smem_u32(sQ + swz<D>(warp * 16 + (lane & 15), kk * 2 + (lane >> 4))));

  float oacc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) oacc[i][0] = oacc[i][1] = oacc[i][2] = oacc[i][3] = 0.f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  const int row_a = q0 + warp * 16 + (lane >> 2);  // local query rows
  const int row_b = row_a + 8;
  const int grow_a = q_off + row_a, grow_b = q_off + row_b;  // global positions

  int stage = 0;
  while (tile < ntiles) {
    const int nxt = next_needed(tile + 1);
    if (nxt < ntiles) load_kv(nxt, stage ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();

    const __nv_bfloat16* cK = sK + stage * 64 * D;
    const __nv_bfloat16* cV = sV + stage * 64 * D;
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int n2 = 0; n2 < 4; ++n2) {
        uint32_t b[4];
        ldsm_x4(b, smem_u32(cK + swz<D>(n2 * 16 + (lane & 7) + ((lane >> 4) << 3), kk * 2 + ((lane >> 3) & 1))));
        mma16816(s[2 * n2], qf[kk], b[0], b[1]);
        mma16816(s[2 * n2 + 1], qf[kk], b[2], b[3]);
      }
    }
    // mask + online softmax (log2 domain)
    const int j0 = tile * 64;
    float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int j = j0 + nt * 8 + 2 * (lane & 3) + e;
        const int ke = j < Tk ? __ldg(kend + j) : -1;
        const bool va = row_a < Tq && j <= grow_a && grow_a < ke;
        const bool vb = row_b < Tq && j <= grow_b && grow_b < ke;
        s[nt][e] = va ? s[nt][e] * scale_log2 : -INFINITY;
        s[nt][2 + e] = vb ? s[nt][2 + e] * scale_log2 : -INFINITY;
        mx_a = fmaxf(mx_a, s[nt][e]);
        mx_b = fmaxf(mx_b, s[nt][2 + e]);
      }
    }
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
    const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
    const float use_a = mn_a == -INFINITY ? 0.f : mn_a;
    const float use_b = mn_b == -INFINITY ? 0.f : mn_b;
    const float corr_a = exp2f(m_a - use_a), corr_b = exp2f(m_b - use_b);
    m_a = mn_a;
    m_b = mn_b;
    l_a *= corr_a;
    l_b *= corr_b;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      oacc[i][0] *= corr_a;
      oacc[i][1] *= corr_a;
      oacc[i][2] *= corr_b;
      oacc[i][3] *= corr_b;
    }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      s[nt][0] = exp2f(s[nt][0] - use_a);
      s[nt][1] = exp2f(s[nt][1] - use_a);
      s[nt][2] = exp2f(s[nt][2] - use_b);
      s[nt][3] = exp2f(s[nt][3] - use_b);
      l_a += s[nt][0] + s[nt][1];
      l_b += s[nt][2] + s[nt][3];
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t a[4];
      a[0] = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
      a[1] = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
      a[2] = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      a[3] = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int n2 = 0; n2 < D / 16; ++n2) {
        uint32_t b[4];
        ldsm_x4_t(b, smem_u32(cV + swz<D>(kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3), n2 * 2 + (lane >> 4))));
        mma16816(oacc[2 * n2], a, b[0], b[1]);
        mma16816(oacc[2 * n2 + 1], a, b[2], b[3]);
      }
    }
    __syncthreads();
    tile = nxt;
    stage ^= 1;
  }
  cp_async_wait<0>();

  l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
  const float inv_a = l_a > 0.f ? 1.f / l_a : 0.f;
  const float inv_b = l_b > 0.f ? 1.f / l_b : 0.f;
#pragma unroll
  for (int nd = 0; nd < D / 8; ++nd) {
    const int col = h * D + nd * 8 + 2 * (lane & 3);
    if (row_a < Tq)
      *reinterpret_cast<uint32_t*>(o + (int64_t)row_a * ldo + col) =
          pack_bf16x2(oacc[nd][0] * inv_a, oacc[nd][1] * inv_a);
    if (row_b < Tq)
      *reinterpret_cast<uint32_t*>(o + (int64_t)row_b * ldo + col) =
          pack_bf16x2(oacc[nd][2] * inv_b, oacc[nd][3] * inv_b);
  }
  if ((lane & 3) == 0) {
    if (row_a < Tq) lse[(int64_t)h * Tq + row_a] = l_a > 0.f ? (m_a + log2f(l_a)) / kLog2e : -INFINITY;
    if (row_b < Tq) lse[(int64_t)h * Tq + row_b] = l_b > 0.f ? (m_b + log2f(l_b)) / kLog2e : -INFINITY;
  }
}

// delta[h, i] = sum_d dO[i, h, d] * O[i, h, d]
template <int D>
__global__ void attn_bwd_pre_kernel(const __nv_bfloat16* __restrict__ dout, int64_t lddo,
                                    const __nv_bfloat16* __restrict__ out, int64_t ldo,
                                    float* __restrict__ delta, int T, int Hq) {
  const int64_t gw = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (gw >= (int64_t)T * Hq) return;
  const int i = gw / Hq, h = gw % Hq;
  const __nv_bfloat16* a = dout + (int64_t)i * lddo + h * D;
  const __nv_bfloat16* b = out + (int64_t)i * ldo + h * D;
  float acc = 0.f;
#pragma unroll
  for (int d = lane * 4; d < D; d += 128) {
    uint2 av = *reinterpret_cast<const uint2*>(a + d);
    uint2 bv = *reinterpret_cast<const uint2*>(b + d);
    const __nv_bfloat16* ae = reinterpret_cast<const __nv_bfloat16*>(&av);
    const __nv_bfloat16* be = reinterpret_cast<const __nv_bfloat16*>(&bv);
#pragma unroll
    for (int e = 0; e < 4; ++e) acc += bf2f(ae[e]) * bf2f(be[e]);
  }
  acc = warp_sum(acc);
  if (lane == 0) delta[(int64_t)h * T + i] = acc;
}

// ----------------------------------------------------------------------------
// Backward: CTA = 128 keys x one kv head (8 warps x 16 keys).  Iterates over
// the q heads of the GQA group and the 32-query tiles that can see the keys.
// dK, dV accumulate in registers; dQ is accumulated with vector fp32 atomics.
// ----------------------------------------------------------------------------
constexpr int BWD_KEYS = 128;
constexpr int BWD_Q = 32;
constexpr int DS_LD = 40;  // padded row (elements) of the dS^T tile: conflict-free ldmatrix

template <int D>
__global__ void __launch_bounds__(256, 1) attn_bwd_kernel(
    const __nv_bfloat16* __restrict__ q, int64_t ldq, const __nv_bfloat16* __restrict__ k,
    int64_t ldk, const __nv_bfloat16* __restrict__ v, int64_t ldv,
    const __nv_bfloat16* __restrict__ dout, int64_t lddo, const float* __restrict__ lse,
    const float* __restrict__ delta, const int* __restrict__ kend,
    const int* __restrict__ units, float* __restrict__ dq_acc, float* __restrict__ dk_acc,
    float* __restrict__ dv_acc, int Tq, int Tk, int q_off, int Hq, int Hkv, float scale) {
  // q tiles of the work units are local query tiles (global position q_off + row)
  static_assert(D == 128, "head_dim 128");
  constexpr int CH = D / 8;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __nv_bfloat16* sK = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  __nv_bfloat16* sV = sK + BWD_KEYS * D;
  __nv_bfloat16* sQ = sV + BWD_KEYS * D;      // 2 stages x 32 x D
  __nv_bfloat16* sdO = sQ + 2 * BWD_Q * D;    // 2 stages x 32 x D
  __nv_bfloat16* sdS = sdO + 2 * BWD_Q * D;   // 128 x DS_LD
  float* sL = reinterpret_cast<float*>(sdS + BWD_KEYS * DS_LD);  // 2 x 32 (log2 units)
  float* sDl = sL + 2 * BWD_Q;                                     // 2 x 32

  // work unit: (key block, first q tile, end q tile); the host splits the
  // query range of heavily attended key blocks (shared prompts) into units
  const int kb = units[3 * blockIdx.x], qt_lo = units[3 * blockIdx.x + 1], qt_hi = units[3 * blockIdx.x + 2];
  // a unit outside the sequence (a malformed work list) is skipped, never read
  if (kb < 0 || (int64_t)kb * BWD_KEYS >= Tk || qt_lo < 0 || (int64_t)qt_lo * BWD_Q >= Tq) return;
  const int hk = blockIdx.y;
  const int G = Hq / Hkv;
  const int j0 = kb * BWD_KEYS;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const float scale_log2 = scale * kLog2e;

  // K, V tiles
  for (int c = tid; c < BWD_KEYS * CH; c += 256) {
    const int r = c / CH, ch = c % CH;
    const int j = j0 + r;
    const int jj = j < Tk ? j : Tk - 1;
    const int nb = j < Tk ? 16 : 0;
    cp_async16(smem_u32(sK + swz<D>(r, ch)), k + (int64_t)jj * ldk + hk * D + ch * 8, nb);
    cp_async16(smem_u32(sV + swz<D>(r, ch)), v + (int64_t)jj * ldv + hk * D + ch * 8, nb);
  }
  cp_async_commit();

  const int qt_begin = qt_lo;
  const int nqt = max(qt_hi - qt_lo, 0);
  const int n_items = nqt * G;

  auto load_item = [&](int n, int st) {
    const int g = n / nqt, qt = qt_begin + n % nqt;
    const int h = hk * G + g;
    const int i0 = qt * BWD_Q;
    for (int c = tid; c < BWD_Q * CH; c += 256) {
      const int r = c / CH, ch = c % CH;
      const int i = i0 + r;
      const int ii = i < Tq ? i : Tq - 1;
      const int nb = i < Tq ? 16 : 0;
      cp_async16(smem_u32(sQ + st * BWD_Q * D + swz<D>(r, ch)), q + (int64_t)ii * ldq + h * D + ch * 8, nb);
      cp_async16(smem_u32(sdO + st * BWD_Q * D + swz<D>(r, ch)), dout + (int64_t)ii * lddo + h * D + ch * 8, nb);
    }
    if (tid < BWD_Q) {
      const int i = i0 + tid;
      sL[st * BWD_Q + tid] = i < Tq ? lse[(int64_t)h * Tq + i] * kLog2e : INFINITY;
      sDl[st * BWD_Q + tid] = i < Tq ? delta[(int64_t)h * Tq + i] : 0.f;
    }
  };

  if (n_items > 0) load_item(0, 0);
  cp_async_commit();
  if (n_items > 1) load_item(1, 1);
  cp_async_commit();

  float dkacc[D / 8][4], dvacc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dkacc[i][e] = dvacc[i][e] = 0.f;

  const int kr0 = warp * 16 + (lane >> 2);  // local key rows owned by this thread
  const int kr1 = kr0 + 8;
  const int ke0 = (j0 + kr0 < Tk) ? __ldg(kend + j0 + kr0) : -1;
  const int ke1 = (j0 + kr1 < Tk) ? __ldg(kend + j0 + kr1) : -1;

  for (int n = 0; n < n_items; ++n) {
    const int st = n & 1;
    const int g = n / nqt, qt = qt_begin + n % nqt;
    const int h = hk * G + g;
    const int i0 = qt * BWD_Q;
    cp_async_wait<1>();
    __syncthreads();
    const __nv_bfloat16* cQ = sQ + st * BWD_Q * D;
    const __nv_bfloat16* cdO = sdO + st * BWD_Q * D;
    const float* cL = sL + st * BWD_Q;
    const float* cDl = sDl + st * BWD_Q;

    // S^T = K_w Q^T and dP^T = V_w dO^T  (16 keys x 32 queries per warp)
    float sT[4][4], dpT[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) sT[i][e] = dpT[i][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t ak[4], av[4];
      ldsm_x4(ak, smem_u32(sK + swz<D>(warp * 16 + (lane & 15), kk * 2 + (lane >> 4))));
      ldsm_x4(av, smem_u32(sV + swz<D>(warp * 16 + (lane & 15), kk * 2 + (lane >> 4))));
#pragma unroll
      for (int n2 = 0; n2 < 2; ++n2) {
        uint32_t bq[4], bo[4];
        const int row = n2 * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int chk = kk * 2 + ((lane >> 3) & 1);
        ldsm_x4(bq, smem_u32(cQ + swz<D>(row, chk)));
        ldsm_x4(bo, smem_u32(cdO + swz<D>(row, chk)));
        mma16816(sT[2 * n2], ak, bq[0], bq[1]);
        mma16816(sT[2 * n2 + 1], ak, bq[2], bq[3]);
        mma16816(dpT[2 * n2], av, bo[0], bo[1]);
        mma16816(dpT[2 * n2 + 1], av, bo[2], bo[3]);
      }
    }
    // P^T and dS^T
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int ql = nt * 8 + 2 * (lane & 3) + e;
        const int i = i0 + ql;  // local query row
        const int gi = q_off + i;  // its global position
        const float L = cL[ql], dl = cDl[ql];
        const int jj0 = j0 + kr0, jj1 = j0 + kr1;
        const bool v0 = i < Tq && jj0 <= gi && gi < ke0;
        const bool v1 = i < Tq && jj1 <= gi && gi < ke1;
        const float p0 = v0 ? exp2f(sT[nt][e] * scale_log2 - L) : 0.f;
        const float p1 = v1 ? exp2f(sT[nt][2 + e] * scale_log2 - L) : 0.f;
        sT[nt][e] = p0;
        sT[nt][2 + e] = p1;
        dpT[nt][e] = p0 * (dpT[nt][e] - dl);
        dpT[nt][2 + e] = p1 * (dpT[nt][2 + e] - dl);
      }
    }
    // dV += P^T dO ; dK += dS^T Q  (k-dim = 32 queries, 2 k-steps)
#pragma unroll
    for (int kq = 0; kq < 2; ++kq) {
      uint32_t ap[4], ads[4];
      ap[0] = pack_bf16x2(sT[2 * kq][0], sT[2 * kq][1]);
      ap[1] = pack_bf16x2(sT[2 * kq][2], sT[2 * kq][3]);
      ap[2] = pack_bf16x2(sT[2 * kq + 1][0], sT[2 * kq + 1][1]);
      ap[3] = pack_bf16x2(sT[2 * kq + 1][2], sT[2 * kq + 1][3]);
      ads[0] = pack_bf16x2(dpT[2 * kq][0], dpT[2 * kq][1]);
      ads[1] = pack_bf16x2(dpT[2 * kq][2], dpT[2 * kq][3]);
      ads[2] = pack_bf16x2(dpT[2 * kq + 1][0], dpT[2 * kq + 1][1]);
      ads[3] = pack_bf16x2(dpT[2 * kq + 1][2], dpT[2 * kq + 1][3]);
#pragma unroll
      for (int n2 = 0; n2 < D / 16; ++n2) {
        uint32_t bo[4], bq[4];
        const int row = kq * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int chk = n2 * 2 + (lane >> 4);
        ldsm_x4_t(bo, smem_u32(cdO + swz<D>(row, chk)));
        ldsm_x4_t(bq, smem_u32(cQ + swz<D>(row, chk)));
        mma16816(dvacc[2 * n2], ap, bo[0], bo[1]);
        mma16816(dvacc[2 * n2 + 1], ap, bo[2], bo[3]);
        mma16816(dkacc[2 * n2], ads, bq[0], bq[1]);
        mma16816(dkacc[2 * n2 + 1], ads, bq[2], bq[3]);
      }
    }
    // stage dS^T (bf16) for the dQ product
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const int col = nt * 8 + 2 * (lane & 3);
      *reinterpret_cast<uint32_t*>(sdS + kr0 * DS_LD + col) = pack_bf16x2(dpT[nt][0], dpT[nt][1]);
      *reinterpret_cast<uint32_t*>(sdS + kr1 * DS_LD + col) = pack_bf16x2(dpT[nt][2], dpT[nt][3]);
    }
    __syncthreads();
    // prefetch item n+2 into this stage (Q/dO of stage st are no longer read)
    if (n + 2 < n_items) load_item(n + 2, st);
    cp_async_commit();

    // dQ (32 x D) += dS (32 x 128) K (128 x D): warp w owns columns [16w, 16w+16)
    float dqa[2][2][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int b = 0; b < 2; ++b)
#pragma unroll
        for (int e = 0; e < 4; ++e) dqa[a][b][e] = 0.f;
#pragma unroll
    for (int kj = 0; kj < BWD_KEYS / 16; ++kj) {
      uint32_t bk[4];
      ldsm_x4_t(bk, smem_u32(sK + swz<D>(kj * 16 + (lane & 7) + (((lane >> 3) & 1) << 3), warp * 2 + (lane >> 4))));
#pragma unroll
      for (int mq = 0; mq < 2; ++mq) {
        uint32_t a[4];
        const int mi = lane >> 3;
        const int krow = kj * 16 + (lane & 7) + ((mi >> 1) << 3);
        const int qcol = mq * 16 + ((mi & 1) << 3);
        ldsm_x4_t(a, smem_u32(sdS + krow * DS_LD + qcol));
        mma16816(dqa[mq][0], a, bk[0], bk[1]);
        mma16816(dqa[mq][1], a, bk[2], bk[3]);
      }
    }
#pragma unroll
    for (int mq = 0; mq < 2; ++mq) {
      const int ia = i0 + mq * 16 + (lane >> 2);
      const int ib = ia + 8;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int col = h * D + warp * 16 + nt * 8 + 2 * (lane & 3);
        if (ia < Tq) red_add_v2(dq_acc + (int64_t)ia * Hq * D + col, dqa[mq][nt][0] * scale, dqa[mq][nt][1] * scale);
        if (ib < Tq) red_add_v2(dq_acc + (int64_t)ib * Hq * D + col, dqa[mq][nt][2] * scale, dqa[mq][nt][3] * scale);
      }
    }
  }
  cp_async_wait<0>();

  // accumulate dK (scaled) and dV for this warp's 16 keys (several units may
  // cover the same key block)
  const int ja = j0 + kr0, jb = j0 + kr1;
#pragma unroll
  for (int nd = 0; nd < D / 8; ++nd) {
    const int col = hk * D + nd * 8 + 2 * (lane & 3);
    if (ja < Tk) {
      red_add_v2(dk_acc + (int64_t)ja * Hkv * D + col, dkacc[nd][0] * scale, dkacc[nd][1] * scale);
      red_add_v2(dv_acc + (int64_t)ja * Hkv * D + col, dvacc[nd][0], dvacc[nd][1]);
    }
    if (jb < Tk) {
      red_add_v2(dk_acc + (int64_t)jb * Hkv * D + col, dkacc[nd][2] * scale, dkacc[nd][3] * scale);
      red_add_v2(dv_acc + (int64_t)jb * Hkv * D + col, dvacc[nd][2], dvacc[nd][3]);
    }
  }
}

static void check_view(const torch::Tensor& t, int64_t T, int64_t H, int64_t D, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16, name, ": bf16 CUDA tensor expected");
  TORCH_CHECK(t.dim() == 3 && t.size(0) == T && t.size(1) == H && t.size(2) == D, name, ": shape");
  TORCH_CHECK(t.stride(2) == 1 && t.stride(1) == D, name, ": heads must be packed");
  TORCH_CHECK(t.stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(t.data_ptr()) % 16) == 0,
              name, ": rows must be 16-byte aligned");
}

// q [Tq, Hq, D] (local queries at global positions q_off + row), k/v [Tk, Hkv, D]
// (row-strided views allowed); kend [Tk] int32; tile_kmax [ceil(Tk/64)] int32.
// Returns o [Tq, Hq, D], lse [Hq, Tq].
std::vector<torch::Tensor> attn_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                    torch::Tensor kend, torch::Tensor tile_kmax, double scale, int64_t q_off) {
  const int64_t Tq = q.size(0), Hq = q.size(1), D = q.size(2), Tk = k.size(0), Hkv = k.size(1);
  TORCH_CHECK(D == 128, "attention kernel supports head_dim 128");
  TORCH_CHECK(Hq % Hkv == 0);
  TORCH_CHECK(q_off >= 0 && q_off + Tq <= Tk, "query range must lie inside the key range");
  check_view(q, Tq, Hq, D, "q");
  check_view(k, Tk, Hkv, D, "k");
  check_view(v, Tk, Hkv, D, "v");
  TORCH_CHECK(kend.scalar_type() == at::kInt && kend.numel() == Tk && kend.is_contiguous());
  TORCH_CHECK(tile_kmax.scalar_type() == at::kInt && tile_kmax.numel() >= (Tk + 63) / 64);
  auto o = torch::empty({Tq, Hq, D}, q.options());
  auto lse = torch::empty({Hq, Tq}, q.options().dtype(at::kFloat));
  if (Tq == 0) return {o, lse};
  const size_t smem = (64 + 4 * 64) * D * sizeof(__nv_bfloat16);
  auto kern = attn_fwd_kernel<128>;
  ART_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((Tq + 63) / 64, Hq);
  kern<<<grid, 128, smem, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), q.stride(0),
      reinterpret_cast<const __nv_bfloat16*>(k.data_ptr()), k.stride(0),
      reinterpret_cast<const __nv_bfloat16*>(v.data_ptr()), v.stride(0), kend.data_ptr<int>(),
      tile_kmax.data_ptr<int>(), reinterpret_cast<__nv_bfloat16*>(o.data_ptr()), o.stride(0),
      lse.data_ptr<float>(), (int)Tq, (int)Tk, (int)q_off, (int)Hq, (int)Hkv, (float)(scale * kLog2e));
  ART_CUDA_CHECK(cudaGetLastError());
  return {o, lse};
}

// Backward.  units [n, 3] int32 = (key block of 128, local q tile lo, local q tile hi)
// in 32-query tiles.  Returns {dq [Tq,Hq,D], dk [Tk,Hkv,D], dv [Tk,Hkv,D]} fp32.
std::vector<torch::Tensor> attn_bwd(torch::Tensor dout, torch::Tensor q, torch::Tensor k,
                                    torch::Tensor v, torch::Tensor out, torch::Tensor lse,
                                    torch::Tensor kend, torch::Tensor units, double scale, int64_t q_off) {
  const int64_t Tq = q.size(0), Hq = q.size(1), D = q.size(2), Tk = k.size(0), Hkv = k.size(1);
  TORCH_CHECK(D == 128);
  TORCH_CHECK(q_off >= 0 && q_off + Tq <= Tk);
  check_view(q, Tq, Hq, D, "q");
  check_view(k, Tk, Hkv, D, "k");
  check_view(v, Tk, Hkv, D, "v");
  check_view(dout, Tq, Hq, D, "dout");
  check_view(out, Tq, Hq, D, "out");
  TORCH_CHECK(kend.numel() == Tk && lse.numel() == Hq * Tq);
  TORCH_CHECK(units.scalar_type() == at::kInt && units.is_contiguous() && units.dim() == 2 && units.size(1) == 3);
  auto f32 = q.options().dtype(at::kFloat);
  auto dq_acc = torch::zeros({Tq, Hq, D}, f32);
  auto dk_acc = torch::zeros({Tk, Hkv, D}, f32);
  auto dv_acc = torch::zeros({Tk, Hkv, D}, f32);
  const int64_t n_units = units.size(0);
  if (Tq == 0 || n_units == 0) return {dq_acc, dk_acc, dv_acc};
  auto delta = torch::empty({Hq, Tq}, f32);
  auto stream = at::cuda::getCurrentCUDAStream();
  {
    const int64_t warps = Tq * Hq;
    attn_bwd_pre_kernel<128><<<(warps + 7) / 8, 256, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), dout.stride(0),
        reinterpret_cast<const __nv_bfloat16*>(out.data_ptr()), out.stride(0),
        delta.data_ptr<float>(), (int)Tq, (int)Hq);
  }
  const size_t smem = (2 * BWD_KEYS * D + 4 * BWD_Q * D + BWD_KEYS * DS_LD) * sizeof(__nv_bfloat16) +
                      4 * BWD_Q * sizeof(float);
  auto kern = attn_bwd_kernel<128>;
  ART_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((unsigned)n_units, Hkv);
  kern<<<grid, 256, smem, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), q.stride(0),
      reinterpret_cast<const __nv_bfloat16*>(k.data_ptr()), k.stride(0),
      reinterpret_cast<const __nv_bfloat16*>(v.data_ptr()), v.stride(0),
      reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), dout.stride(0), lse.data_ptr<float>(),
      delta.data_ptr<float>(), kend.data_ptr<int>(), units.data_ptr<int>(), dq_acc.data_ptr<float>(),
      dk_acc.data_ptr<float>(), dv_acc.data_ptr<float>(), (int)Tq, (int)Tk, (int)q_off, (int)Hq, (int)Hkv,
      (float)scale);
  ART_CUDA_CHECK(cudaGetLastError());
  return {dq_acc, dk_acc, dv_acc};
}

}  // namespace art

// ============================================================================
// Allocation-free C entry point of the attention backward (declared, with its
// layouts, limits and return codes, in art_noalloc.h).
//
// No counterpart in the reference: it serves callers that cannot allocate
// device memory themselves -- code running inside a host application that owns
// the whole device memory budget (a plugin given fixed buffers), or a
// latency-critical loop that must never enter the CUDA allocator, which can
// synchronise the device.  The caller passes every input and output; the only
// extra memory, the per-(head, query) `delta = sum(dO*O)` vector, lives in the
// fixed file-scope device array below (4 MiB per device, held until exit).
// ============================================================================
namespace {
static __device__ __align__(256) float g_noalloc_delta[ART_NOALLOC_DELTA_MAX];

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// A bf16 operand of `heads` x 128 columns per row: 16-byte base, row stride a
// multiple of 8 elements (16 bytes) covering the row.
bool operand_ok(const void* p, int64_t ld, int heads) {
  return p && aligned16(p) && ld % 8 == 0 && ld >= (int64_t)heads * 128;
}
}  // namespace

extern "C" int art_attn_bwd_noalloc(const void* dout, int64_t lddo, const void* q, int64_t ldq, const void* k,
                                    int64_t ldk, const void* v, int64_t ldv, const void* out, int64_t ldo,
                                    const float* lse, const int* kend, const int* units, int n_units, float* dq,
                                    float* dk, float* dv, int T, int Hq, int Hkv, int D, float scale,
                                    cudaStream_t stream) {
  using namespace art;
  if (D != 128) return ART_NOALLOC_BAD_HEAD_DIM;
  if (T < 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0 || n_units < 0) return ART_NOALLOC_BAD_ARGUMENT;
  if ((int64_t)T * Hq > ART_NOALLOC_DELTA_MAX) return ART_NOALLOC_TOO_LARGE;
  // every check below runs before anything touches the device
  if (!operand_ok(dout, lddo, Hq) || !operand_ok(q, ldq, Hq) || !operand_ok(out, ldo, Hq) ||
      !operand_ok(k, ldk, Hkv) || !operand_ok(v, ldv, Hkv))
    return ART_NOALLOC_BAD_ARGUMENT;
  if (!lse || !kend || !dq || !dk || !dv || (n_units > 0 && !units)) return ART_NOALLOC_BAD_ARGUMENT;
  if (!aligned16(dq) || !aligned16(dk) || !aligned16(dv)) return ART_NOALLOC_BAD_ARGUMENT;
  // The array's name is a host-side stand-in in host code: its device address
  // is looked up here, on the caller's current device, on every call (no
  // cache that a device reset could leave dangling; no allocation).
  void* sym = nullptr;
  if (cudaGetSymbolAddress(&sym, g_noalloc_delta) != cudaSuccess || !sym) return ART_NOALLOC_CUDA_ERROR;
  float* delta = static_cast<float*>(sym);
  const size_t nq = (size_t)T * Hq * D * sizeof(float), nk = (size_t)T * Hkv * D * sizeof(float);
  if (cudaMemsetAsync(dq, 0, nq, stream) != cudaSuccess) return ART_NOALLOC_CUDA_ERROR;
  if (cudaMemsetAsync(dk, 0, nk, stream) != cudaSuccess) return ART_NOALLOC_CUDA_ERROR;
  if (cudaMemsetAsync(dv, 0, nk, stream) != cudaSuccess) return ART_NOALLOC_CUDA_ERROR;
  if (T == 0 || n_units == 0) return ART_NOALLOC_OK;
  // launched through cudaLaunchKernel so that each launch's own status is
  // returned (an earlier, unrelated error pending in the runtime is not
  // reported as this call's failure)
  {
    const int64_t warps = (int64_t)T * Hq;
    const __nv_bfloat16* a0 = reinterpret_cast<const __nv_bfloat16*>(dout);
    const __nv_bfloat16* a2 = reinterpret_cast<const __nv_bfloat16*>(out);
    int64_t a1 = lddo, a3 = ldo;
    float* a4 = delta;
    int a5 = T, a6 = Hq;
    void* args[] = {&a0, &a1, &a2, &a3, &a4, &a5, &a6};
    if (cudaLaunchKernel(reinterpret_cast<const void*>(&attn_bwd_pre_kernel<128>), dim3((unsigned)((warps + 7) / 8)),
                         dim3(256), args, 0, stream) != cudaSuccess)
      return ART_NOALLOC_CUDA_ERROR;
  }
  const size_t smem = (2 * BWD_KEYS * 128 + 4 * BWD_Q * 128 + BWD_KEYS * DS_LD) * sizeof(__nv_bfloat16) +
                      4 * BWD_Q * sizeof(float);
  if (cudaFuncSetAttribute(attn_bwd_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return ART_NOALLOC_CUDA_ERROR;
  {
    const __nv_bfloat16 *pq = reinterpret_cast<const __nv_bfloat16*>(q), *pk = reinterpret_cast<const __nv_bfloat16*>(k),
                        *pv = reinterpret_cast<const __nv_bfloat16*>(v),
                        *pdo = reinterpret_cast<const __nv_bfloat16*>(dout);
    int64_t lq = ldq, lk = ldk, lv = ldv, ld = lddo;
    const float* plse = lse;
    const float* pdelta = delta;
    const int* pkend = kend;
    const int* punits = units;
    float *pdq = dq, *pdk = dk, *pdv = dv;
    int tq = T, tk = T, qoff = 0, hq = Hq, hkv = Hkv;
    float sc = scale;
    void* args[] = {&pq, &lq, &pk, &lk, &pv, &lv, &pdo, &ld, &plse, &pdelta, &pkend, &punits,
                    &pdq, &pdk, &pdv, &tq, &tk, &qoff, &hq, &hkv, &sc};
    if (cudaLaunchKernel(reinterpret_cast<const void*>(&attn_bwd_kernel<128>), dim3((unsigned)n_units, (unsigned)Hkv),
                         dim3(256), args, smem, stream) != cudaSuccess)
      return ART_NOALLOC_CUDA_ERROR;
  }
  return ART_NOALLOC_OK;
}
