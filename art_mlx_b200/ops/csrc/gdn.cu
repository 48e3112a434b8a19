// Gated DeltaNet kernels: the sequential chunk scan of the gated delta rule
// (forward and backward) and the packed tree causal conv + SiLU.
//
// Chunked delta rule, per row r (one sequence x one head), chunk c of C = 64
// tokens, state S [DK x DV] fp32 (the per-chunk operands are produced by
// batched tensor-core GEMMs beforehand):
//
//   U      = U0 - W S                      [C x DV]
//   O      = gq S + QKM U                  [C x DV]   (optional)
//   S_next = gC S + Kd^T U                 [DK x DV]
//
// Backward (reverse over chunks, dS = gradient of S_next):
//
//   dU     = QKM^T dO + Kd dS              (= dU0; dW = -dU S^T outside)
//   dS_prev= gC dS + gq^T dO - W^T dU
//
// Only these recurrences are sequential; every product that contracts over
// DV (dgq = dO S^T, dW, dQKM = dO U^T, dKd = U dS^T, dgC) is batched over all
// chunks outside, so the scan kernels save the state entering each chunk (S)
// and the gradient leaving it (dS) for those GEMMs.
//
// Value columns are independent in both recurrences, so a CTA owns one
// 32-column slice of one row: grid (DV/32, rows).  256 threads; each thread
// holds a 2x4 tile of the [C x 32] products and a (DK/32)x4 tile of the
// [DK x 32] products, reading the chunk operands from shared memory as
// float4 (a quarter-warp shares one operand row -> broadcast).  Chunk c+1's
// operands are fetched with cp.async while chunk c computes: the W/U0 group
// after the first product, the rest after the state update.
//
// The same scan with S0 = [I | 0] and U0 = [0 | U0] yields the affine
// summary [A | B] of a span of chunks (S_out = A S_in + B), the quantity
// context parallelism exchanges between ranks.  `peer_out` lets that call
// store the summary straight into every peer's receive slot over NVLink
// (P2P stores from the CTA that owns the columns), fusing the exchange into
// the scan's epilogue.
//
// Conv: y = silu(sum_m w[:, W-1-m] * x[prev_m(i)]) with prev_0(i) = i and
// prev_m the packed index m positions back in the token's sequence (-1 before
// its start), so a completion's first tokens read the end of its prompt.
// Backward: one pass forms dpre = dy * silu'(pre) and reduces dw per CTA (one
// atomic per tap); a second gathers dx over each token's successors from a
// CSR table (a branch point's last tokens feed every child's first tokens),
// so dx has a single writer and no atomics.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "common.cuh"

namespace art {
namespace {

constexpr int GC = 64;        // chunk length
constexpr int GVS = 32;       // value columns per CTA
constexpr int GTHREADS = 256;

template <int DK>
struct ScanLayout {
  static constexpr int S = 0;                    // [DK][GVS]  state (fwd) / dstate (bwd)
  static constexpr int T1 = S + DK * GVS;        // [GC][DK]   W (fwd) / Kd (bwd)
  static constexpr int T2 = T1 + GC * DK;        // [GC][DK]   gq
  static constexpr int T3 = T2 + GC * DK;        // [GC][DK]   Kd (fwd) / W (bwd)
  static constexpr int QK = T3 + GC * DK;        // [GC][GC]   QKM
  static constexpr int V0 = QK + GC * GC;        // [GC][GVS]  U0 (fwd) / dO buffer 0 (bwd)
  static constexpr int V1 = V0 + GC * GVS;       // [GC][GVS]  U (fwd) / dO buffer 1 (bwd)
  static constexpr int V2 = V1 + GC * GVS;       // [GC][GVS]  dU (bwd)
  static constexpr int TOTAL = V2 + GC * GVS;    // floats
};

// cp.async a [rows x cols] fp32 block (row stride ld floats) into dense smem.
__device__ __forceinline__ void stage(float* dst, const float* src, int rows, int cols, int64_t ld) {
  const int per_row = cols >> 2;
  for (int e = threadIdx.x; e < rows * per_row; e += GTHREADS) {
    const int r = e / per_row, q = e - r * per_row;
    cp_async16(smem_u32(dst + r * cols + (q << 2)), src + r * ld + (q << 2), 16);
  }
}

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }

// acc[a][j] += sum_k A[row_a][k] * B[k][col0 + j]  over k in [0, K), A row-major
// (stride lda), B row-major stride GVS.  Two rows (ra, ra+1), four columns.
template <int K>
__device__ __forceinline__ void mm_rows2(float acc[2][4], const float* A, int lda, int ra, const float* B, int c0) {
#pragma unroll 4
  for (int k = 0; k < K; k += 4) {
    const float4 a0 = ld4(A + ra * lda + k), a1 = ld4(A + (ra + 1) * lda + k);
    const float av0[4] = {a0.x, a0.y, a0.z, a0.w}, av1[4] = {a1.x, a1.y, a1.z, a1.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float4 b = ld4(B + (k + t) * GVS + c0);
      acc[0][0] += av0[t] * b.x; acc[0][1] += av0[t] * b.y; acc[0][2] += av0[t] * b.z; acc[0][3] += av0[t] * b.w;
      acc[1][0] += av1[t] * b.x; acc[1][1] += av1[t] * b.y; acc[1][2] += av1[t] * b.z; acc[1][3] += av1[t] * b.w;
    }
  }
}

// acc[a][j] += sum_i A[i][ra + a] * B[i][c0 + j]  (A read transposed, A row stride lda;
// RA consecutive rows of the result), i in [0, GC).
template <int RA>
__device__ __forceinline__ void mm_trans(float acc[RA][4], const float* A, int lda, int ra, const float* B, int c0) {
#pragma unroll 4
  for (int i = 0; i < GC; ++i) {
    float a[RA];
    if constexpr (RA == 4) {
      const float4 v = ld4(A + i * lda + ra);
      a[0] = v.x; a[1] = v.y; a[2] = v.z; a[3] = v.w;
    } else {
      const float2 v = *reinterpret_cast<const float2*>(A + i * lda + ra);
      a[0] = v.x; a[1] = v.y;
    }
    const float4 b = ld4(B + i * GVS + c0);
#pragma unroll
    for (int r = 0; r < RA; ++r) {
      acc[r][0] += a[r] * b.x; acc[r][1] += a[r] * b.y; acc[r][2] += a[r] * b.z; acc[r][3] += a[r] * b.w;
    }
  }
}

struct ScanArgs {
  const float* gq;    // [R, nc, GC, DK]
  const float* W;     // [R, nc, GC, DK]
  const float* U0;    // [R, nc, GC, DV]
  const float* QKM;   // [R, nc, GC, GC]
  const float* Kd;    // [R, nc, GC, DK]
  const float* gC;    // [R, nc]
  const float* S0;    // [R, DK, DV] or null (zero)
  float* O;           // [R, nc, GC, DV] or null (no output)
  float* S_end;       // [R, DK, DV]
  float* states;      // [R, nc, DK, DV] or null (state entering each chunk)
  float* Usave;       // [R, nc, GC, DV] or null
  const int64_t* peer_out;  // [npeers] base pointers of the peers' summary slots, or null
  int npeers;
  int nc, DV;
};

template <int DK>
__global__ void __launch_bounds__(GTHREADS, 1) gdn_scan_fwd_kernel(ScanArgs a) {
  using L = ScanLayout<DK>;
  constexpr int RK = DK / 32;  // state rows per thread
  extern __shared__ __align__(16) float sm[];
  float* sS = sm + L::S;
  float* sW = sm + L::T1;
  float* sQ = sm + L::T2;
  float* sK = sm + L::T3;
  float* sM = sm + L::QK;
  float* sU0 = sm + L::V0;
  float* sU = sm + L::V1;

  const int tid = threadIdx.x;
  const int col0 = blockIdx.x * GVS;
  const int64_t r = blockIdx.y;
  const int nc = a.nc, DV = a.DV;
  const int ri = (tid >> 3) * 2, ci = (tid & 7) * 4;  // [GC x 32] tiles: rows ri, ri+1
  const int rk = (tid >> 3) * RK;                     // [DK x 32] tiles: rows rk .. rk+RK-1

  // initial state slice
  for (int e = tid; e < DK * (GVS / 4); e += GTHREADS) {
    const int k = e / (GVS / 4), q = (e % (GVS / 4)) * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (a.S0) v = ld4(a.S0 + (r * DK + k) * DV + col0 + q);
    st4(sS + k * GVS + q, v);
  }
  auto chunk_base = [&](int c, int width) -> int64_t { return ((r * nc + c) * GC) * (int64_t)width; };
  // prologue: group A(0) = {W, U0}, group B(0) = {gq, QKM, Kd}
  stage(sW, a.W + chunk_base(0, DK), GC, DK, DK);
  stage(sU0, a.U0 + chunk_base(0, DV) + col0, GC, GVS, DV);
  cp_async_commit();
  stage(sQ, a.gq + chunk_base(0, DK), GC, DK, DK);
  stage(sM, a.QKM + chunk_base(0, GC), GC, GC, GC);
  stage(sK, a.Kd + chunk_base(0, DK), GC, DK, DK);
  cp_async_commit();

  for (int c = 0; c < nc; ++c) {
    cp_async_wait<1>();
    __syncthreads();
    const float gc = a.gC[r * nc + c];
    if (a.states) {
      float* dst = a.states + ((r * nc + c) * DK) * (int64_t)DV + col0;
#pragma unroll
      for (int t = 0; t < RK; ++t) st4(dst + (rk + t) * (int64_t)DV + ci, ld4(sS + (rk + t) * GVS + ci));
    }
    // U = U0 - W S
    float u[2][4] = {};
    mm_rows2<DK>(u, sW, DK, ri, sS, ci);
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const float4 b = ld4(sU0 + (ri + t) * GVS + ci);
      const float4 v = make_float4(b.x - u[t][0], b.y - u[t][1], b.z - u[t][2], b.w - u[t][3]);
      st4(sU + (ri + t) * GVS + ci, v);
      if (a.Usave) st4(a.Usave + chunk_base(c, DV) + (int64_t)(ri + t) * DV + col0 + ci, v);
    }
    __syncthreads();
    if (c + 1 < nc) {
      stage(sW, a.W + chunk_base(c + 1, DK), GC, DK, DK);
      stage(sU0, a.U0 + chunk_base(c + 1, DV) + col0, GC, GVS, DV);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    // O = gq S + QKM U
    if (a.O) {
      float o[2][4] = {};
      mm_rows2<DK>(o, sQ, DK, ri, sS, ci);
      mm_rows2<GC>(o, sM, GC, ri, sU, ci);
#pragma unroll
      for (int t = 0; t < 2; ++t)
        st4(a.O + chunk_base(c, DV) + (int64_t)(ri + t) * DV + col0 + ci,
            make_float4(o[t][0], o[t][1], o[t][2], o[t][3]));
    }
    // S_next = gC S + Kd^T U
    float s[RK][4] = {};
    mm_trans<RK>(s, sK, DK, rk, sU, ci);
#pragma unroll
    for (int t = 0; t < RK; ++t) {
      const float4 old = ld4(sS + (rk + t) * GVS + ci);
      s[t][0] += gc * old.x; s[t][1] += gc * old.y; s[t][2] += gc * old.z; s[t][3] += gc * old.w;
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < RK; ++t) st4(sS + (rk + t) * GVS + ci, make_float4(s[t][0], s[t][1], s[t][2], s[t][3]));
    if (c + 1 < nc) {
      stage(sQ, a.gq + chunk_base(c + 1, DK), GC, DK, DK);
      stage(sM, a.QKM + chunk_base(c + 1, GC), GC, GC, GC);
      stage(sK, a.Kd + chunk_base(c + 1, DK), GC, DK, DK);
      cp_async_commit();
    }
  }
  __syncthreads();
  // final state (each thread writes the rows it updated last)
#pragma unroll
  for (int t = 0; t < RK; ++t) {
    const float4 v = ld4(sS + (rk + t) * GVS + ci);
    const int64_t off = (r * DK + rk + t) * (int64_t)DV + col0 + ci;
    st4(a.S_end + off, v);
    for (int p = 0; p < a.npeers; ++p)  // fused exchange: the same slice into every peer's slot
      st4(reinterpret_cast<float*>(a.peer_out[p]) + off, v);
  }
  if (a.npeers) __threadfence_system();
}

struct ScanBwdArgs {
  const float* dO;     // [R, nc, GC, DV] or null (zero)
  const float* dS_end; // [R, DK, DV] or null (zero)
  const float* gq;
  const float* W;
  const float* QKM;
  const float* Kd;
  const float* gC;
  float* dU;           // [R, nc, GC, DV]
  float* dSa;          // [R, nc, DK, DV] gradient of the state leaving each chunk
  float* dS0;          // [R, DK, DV]
  int nc, DV;
};

template <int DK>
__global__ void __launch_bounds__(GTHREADS, 1) gdn_scan_bwd_kernel(ScanBwdArgs a) {
  using L = ScanLayout<DK>;
  constexpr int RK = DK / 32;
  extern __shared__ __align__(16) float sm[];
  float* sD = sm + L::S;     // dS
  float* sK = sm + L::T1;    // Kd
  float* sQ = sm + L::T2;    // gq
  float* sW = sm + L::T3;    // W
  float* sM = sm + L::QK;    // QKM
  float* const sdO0 = sm + L::V0;
  float* const sdO1 = sm + L::V1;
  float* sdU = sm + L::V2;

  const int tid = threadIdx.x;
  const int col0 = blockIdx.x * GVS;
  const int64_t r = blockIdx.y;
  const int nc = a.nc, DV = a.DV;
  const int ri = (tid >> 3) * 2, ci = (tid & 7) * 4;
  const int rk = (tid >> 3) * RK;
  const bool has_do = a.dO != nullptr;

  for (int e = tid; e < DK * (GVS / 4); e += GTHREADS) {
    const int k = e / (GVS / 4), q = (e % (GVS / 4)) * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (a.dS_end) v = ld4(a.dS_end + (r * DK + k) * DV + col0 + q);
    st4(sD + k * GVS + q, v);
  }
  if (!has_do) {
    for (int e = tid; e < GC * GVS; e += GTHREADS) sdO0[e] = 0.f;
  }
  auto chunk_base = [&](int c, int width) -> int64_t { return ((r * nc + c) * GC) * (int64_t)width; };
  // group A(c) = {QKM, Kd, dO}, group B(c) = {gq, W}
  const int last = nc - 1;
  stage(sM, a.QKM + chunk_base(last, GC), GC, GC, GC);
  stage(sK, a.Kd + chunk_base(last, DK), GC, DK, DK);
  if (has_do) stage((last & 1) ? sdO1 : sdO0, a.dO + chunk_base(last, DV) + col0, GC, GVS, DV);
  cp_async_commit();
  stage(sQ, a.gq + chunk_base(last, DK), GC, DK, DK);
  stage(sW, a.W + chunk_base(last, DK), GC, DK, DK);
  cp_async_commit();

  for (int c = last; c >= 0; --c) {
    cp_async_wait<1>();
    __syncthreads();
    const float gc = a.gC[r * nc + c];
    const float* dOc = (has_do && (c & 1)) ? sdO1 : sdO0;
    // the gradient leaving chunk c
    {
      float* dst = a.dSa + ((r * nc + c) * DK) * (int64_t)DV + col0;
#pragma unroll
      for (int t = 0; t < RK; ++t) st4(dst + (rk + t) * (int64_t)DV + ci, ld4(sD + (rk + t) * GVS + ci));
    }
    // dU = QKM^T dO + Kd dS
    float u[2][4] = {};
    if (has_do) mm_trans<2>(u, sM, GC, ri, dOc, ci);
    mm_rows2<DK>(u, sK, DK, ri, sD, ci);
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const float4 v = make_float4(u[t][0], u[t][1], u[t][2], u[t][3]);
      st4(sdU + (ri + t) * GVS + ci, v);
      st4(a.dU + chunk_base(c, DV) + (int64_t)(ri + t) * DV + col0 + ci, v);
    }
    __syncthreads();
    if (c > 0) {
      stage(sM, a.QKM + chunk_base(c - 1, GC), GC, GC, GC);
      stage(sK, a.Kd + chunk_base(c - 1, DK), GC, DK, DK);
      if (has_do) stage(((c - 1) & 1) ? sdO1 : sdO0, a.dO + chunk_base(c - 1, DV) + col0, GC, GVS, DV);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    // dS_prev = gC dS + gq^T dO - W^T dU
    float s[RK][4] = {};
    if (has_do) mm_trans<RK>(s, sQ, DK, rk, dOc, ci);
    float w[RK][4] = {};
    mm_trans<RK>(w, sW, DK, rk, sdU, ci);
#pragma unroll
    for (int t = 0; t < RK; ++t) {
      const float4 old = ld4(sD + (rk + t) * GVS + ci);
      s[t][0] += gc * old.x - w[t][0]; s[t][1] += gc * old.y - w[t][1];
      s[t][2] += gc * old.z - w[t][2]; s[t][3] += gc * old.w - w[t][3];
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < RK; ++t) st4(sD + (rk + t) * GVS + ci, make_float4(s[t][0], s[t][1], s[t][2], s[t][3]));
    if (c > 0) {
      stage(sQ, a.gq + chunk_base(c - 1, DK), GC, DK, DK);
      stage(sW, a.W + chunk_base(c - 1, DK), GC, DK, DK);
      cp_async_commit();
    }
  }
  __syncthreads();
#pragma unroll
  for (int t = 0; t < RK; ++t)
    st4(a.dS0 + (r * DK + rk + t) * (int64_t)DV + col0 + ci, ld4(sD + (rk + t) * GVS + ci));
}

// ---------------------------------------------------------------- conv
constexpr int CONV_ROWS = 64;
constexpr int CONV_THREADS = 128;
constexpr int CONV_MAXW = 8;

// Taps reversed: wr[t] multiplies the input t positions back (wr[0] = current).
template <typename T>
__device__ __forceinline__ void load_taps(float wr[CONV_MAXW], const T* w, int ch, int W) {
#pragma unroll
  for (int t = 0; t < CONV_MAXW; ++t) wr[t] = t < W ? static_cast<float>(w[(int64_t)ch * W + (W - 1 - t)]) : 0.f;
}

template <typename T>
__device__ __forceinline__ float conv_pre(const T* x, const int64_t* prev, const float wr[CONV_MAXW], int64_t i,
                                          int ch, int C, int W, float xs[CONV_MAXW]) {
  xs[0] = static_cast<float>(x[i * C + ch]);
  float acc = wr[0] * xs[0];
#pragma unroll
  for (int t = 1; t < CONV_MAXW; ++t) {
    xs[t] = 0.f;
    if (t < W) {
      const int64_t j = prev[i * (W - 1) + (t - 1)];
      if (j >= 0) xs[t] = static_cast<float>(x[j * C + ch]);
      acc += wr[t] * xs[t];
    }
  }
  return acc;
}

template <typename T>
__global__ void __launch_bounds__(CONV_THREADS) gdn_conv_fwd_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                                     const int64_t* __restrict__ prev,
                                                                     float* __restrict__ y, int64_t rows, int C, int W) {
  const int ch = blockIdx.x * CONV_THREADS + threadIdx.x;
  if (ch >= C) return;
  float wr[CONV_MAXW], xs[CONV_MAXW];
  load_taps(wr, w, ch, W);
  const int64_t i0 = (int64_t)blockIdx.y * CONV_ROWS;
  const int64_t i1 = i0 + CONV_ROWS < rows ? i0 + CONV_ROWS : rows;
  for (int64_t i = i0; i < i1; ++i) {
    const float pre = conv_pre(x, prev, wr, i, ch, C, W, xs);
    y[i * C + ch] = pre / (1.f + __expf(-pre));
  }
}

// dpre = dy * silu'(pre); dw reduced over the CTA's rows, one atomic per tap.
template <typename T>
__global__ void __launch_bounds__(CONV_THREADS) gdn_conv_dpre_kernel(const float* __restrict__ dy, const T* __restrict__ x,
                                                                      const T* __restrict__ w,
                                                                      const int64_t* __restrict__ prev,
                                                                      float* __restrict__ dpre, float* __restrict__ dw,
                                                                      int64_t rows, int C, int W) {
  const int ch = blockIdx.x * CONV_THREADS + threadIdx.x;
  if (ch >= C) return;
  float wr[CONV_MAXW], xs[CONV_MAXW], gw[CONV_MAXW];
  load_taps(wr, w, ch, W);
#pragma unroll
  for (int t = 0; t < CONV_MAXW; ++t) gw[t] = 0.f;
  const int64_t i0 = (int64_t)blockIdx.y * CONV_ROWS;
  const int64_t i1 = i0 + CONV_ROWS < rows ? i0 + CONV_ROWS : rows;
  for (int64_t i = i0; i < i1; ++i) {
    const float pre = conv_pre(x, prev, wr, i, ch, C, W, xs);
    const float sg = 1.f / (1.f + __expf(-pre));
    const float dp = dy[i * C + ch] * sg * (1.f + pre * (1.f - sg));
    dpre[i * C + ch] = dp;
#pragma unroll
    for (int t = 0; t < CONV_MAXW; ++t) gw[t] += dp * xs[t];
  }
#pragma unroll
  for (int t = 0; t < CONV_MAXW; ++t)
    if (t < W) atomicAdd(dw + (int64_t)ch * W + (W - 1 - t), gw[t]);
}

// dx[j] = sum over j's successors (i, tap t) of wr[t] * dpre[i]; the CSR
// (succ_ptr, succ_idx, succ_tap) lists them, the direct term (j, 0) included.
template <typename T>
__global__ void __launch_bounds__(CONV_THREADS) gdn_conv_dx_kernel(const float* __restrict__ dpre, const T* __restrict__ w,
                                                                    const int64_t* __restrict__ succ_ptr,
                                                                    const int64_t* __restrict__ succ_idx,
                                                                    const int8_t* __restrict__ succ_tap,
                                                                    T* __restrict__ dx, int64_t rows, int C, int W) {
  const int ch = blockIdx.x * CONV_THREADS + threadIdx.x;
  if (ch >= C) return;
  float wr[CONV_MAXW];
  load_taps(wr, w, ch, W);
  const int64_t j0 = (int64_t)blockIdx.y * CONV_ROWS;
  const int64_t j1 = j0 + CONV_ROWS < rows ? j0 + CONV_ROWS : rows;
  for (int64_t j = j0; j < j1; ++j) {
    float acc = 0.f;
    for (int64_t e = succ_ptr[j]; e < succ_ptr[j + 1]; ++e) {
      const int t = succ_tap[e];
      float wt = 0.f;
#pragma unroll
      for (int q = 0; q < CONV_MAXW; ++q) wt = q == t ? wr[q] : wt;
      acc += wt * dpre[succ_idx[e] * C + ch];
    }
    dx[j * C + ch] = static_cast<T>(acc);
  }
}

void check_f32(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kFloat32 && t.is_contiguous(), name,
              " must be a contiguous fp32 CUDA tensor");
}

template <int DK>
void launch_fwd(const ScanArgs& a, int R, cudaStream_t st) {
  const size_t smem = ScanLayout<DK>::TOTAL * sizeof(float);
  auto kern = gdn_scan_fwd_kernel<DK>;
  ART_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  kern<<<dim3(a.DV / GVS, R), GTHREADS, smem, st>>>(a);
  ART_CUDA_CHECK(cudaGetLastError());
}

template <int DK>
void launch_bwd(const ScanBwdArgs& a, int R, cudaStream_t st) {
  const size_t smem = ScanLayout<DK>::TOTAL * sizeof(float);
  auto kern = gdn_scan_bwd_kernel<DK>;
  ART_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  kern<<<dim3(a.DV / GVS, R), GTHREADS, smem, st>>>(a);
  ART_CUDA_CHECK(cudaGetLastError());
}

}  // namespace

// Forward scan.  Returns [O (empty unless want_out), S_end, states (empty unless
// save), U (empty unless save)].  `peer_out` (int64 pointers, optional): the
// final state is also stored at each address (same [R, DK, DV] layout).
std::vector<torch::Tensor> gdn_scan_fwd(torch::Tensor gq, torch::Tensor W, torch::Tensor U0, torch::Tensor QKM,
                                        torch::Tensor Kd, torch::Tensor gC, c10::optional<torch::Tensor> S0,
                                        bool want_out, bool save, c10::optional<torch::Tensor> peer_out) {
  for (auto* p : {&gq, &W, &U0, &QKM, &Kd, &gC}) check_f32(*p, "gdn_scan_fwd operand");
  TORCH_CHECK(W.dim() == 4 && W.size(2) == GC, "W must be [R, nc, 64, DK]");
  const int64_t R = W.size(0), nc = W.size(1), DK = W.size(3), DV = U0.size(3);
  TORCH_CHECK(DK == 64 || DK == 128, "key head dim must be 64 or 128");
  TORCH_CHECK(DV % GVS == 0, "value width must be a multiple of 32");
  TORCH_CHECK(gq.sizes() == W.sizes() && Kd.sizes() == W.sizes(), "gq/Kd shape mismatch");
  TORCH_CHECK(U0.size(0) == R && U0.size(1) == nc && U0.size(2) == GC, "U0 shape mismatch");
  TORCH_CHECK(QKM.size(0) == R && QKM.size(1) == nc && QKM.size(2) == GC && QKM.size(3) == GC, "QKM shape mismatch");
  TORCH_CHECK(gC.numel() == R * nc, "gC shape mismatch");
  TORCH_CHECK(R <= 65535, "too many rows");
  auto opts = W.options();
  torch::Tensor O = want_out ? torch::empty({R, nc, GC, DV}, opts) : torch::empty({0}, opts);
  torch::Tensor S_end = torch::empty({R, DK, DV}, opts);
  torch::Tensor states = save ? torch::empty({R, nc, DK, DV}, opts) : torch::empty({0}, opts);
  torch::Tensor Us = save ? torch::empty({R, nc, GC, DV}, opts) : torch::empty({0}, opts);
  ScanArgs a{};
  a.gq = gq.data_ptr<float>();
  a.W = W.data_ptr<float>();
  a.U0 = U0.data_ptr<float>();
  a.QKM = QKM.data_ptr<float>();
  a.Kd = Kd.data_ptr<float>();
  a.gC = gC.data_ptr<float>();
  if (S0.has_value()) {
    check_f32(*S0, "S0");
    TORCH_CHECK(S0->numel() == R * DK * DV, "S0 shape mismatch");
    a.S0 = S0->data_ptr<float>();
  }
  a.O = want_out ? O.data_ptr<float>() : nullptr;
  a.S_end = S_end.data_ptr<float>();
  a.states = save ? states.data_ptr<float>() : nullptr;
  a.Usave = save ? Us.data_ptr<float>() : nullptr;
  if (peer_out.has_value() && peer_out->numel() > 0) {
    TORCH_CHECK(peer_out->is_cuda() && peer_out->scalar_type() == torch::kInt64, "peer_out must be int64 on device");
    a.peer_out = peer_out->data_ptr<int64_t>();
    a.npeers = (int)peer_out->numel();
  }
  a.nc = (int)nc;
  a.DV = (int)DV;
  if (nc > 0) {
    auto st = at::cuda::getCurrentCUDAStream();
    if (DK == 128) launch_fwd<128>(a, (int)R, st);
    else launch_fwd<64>(a, (int)R, st);
  }
  return {O, S_end, states, Us};
}

// Backward scan.  Returns [dU, dSa, dS0].
std::vector<torch::Tensor> gdn_scan_bwd(c10::optional<torch::Tensor> dO, c10::optional<torch::Tensor> dS_end,
                                        torch::Tensor gq, torch::Tensor W, torch::Tensor QKM, torch::Tensor Kd,
                                        torch::Tensor gC, int64_t DV) {
  for (auto* p : {&gq, &W, &QKM, &Kd, &gC}) check_f32(*p, "gdn_scan_bwd operand");
  const int64_t R = W.size(0), nc = W.size(1), DK = W.size(3);
  TORCH_CHECK(DK == 64 || DK == 128, "key head dim must be 64 or 128");
  TORCH_CHECK(DV % GVS == 0, "value width must be a multiple of 32");
  auto opts = W.options();
  torch::Tensor dU = torch::empty({R, nc, GC, DV}, opts);
  torch::Tensor dSa = torch::empty({R, nc, DK, DV}, opts);
  torch::Tensor dS0 = torch::empty({R, DK, DV}, opts);
  ScanBwdArgs a{};
  if (dO.has_value()) {
    check_f32(*dO, "dO");
    TORCH_CHECK(dO->numel() == R * nc * GC * DV, "dO shape mismatch");
    a.dO = dO->data_ptr<float>();
  }
  if (dS_end.has_value()) {
    check_f32(*dS_end, "dS_end");
    TORCH_CHECK(dS_end->numel() == R * DK * DV, "dS_end shape mismatch");
    a.dS_end = dS_end->data_ptr<float>();
  }
  a.gq = gq.data_ptr<float>();
  a.W = W.data_ptr<float>();
  a.QKM = QKM.data_ptr<float>();
  a.Kd = Kd.data_ptr<float>();
  a.gC = gC.data_ptr<float>();
  a.dU = dU.data_ptr<float>();
  a.dSa = dSa.data_ptr<float>();
  a.dS0 = dS0.data_ptr<float>();
  a.nc = (int)nc;
  a.DV = (int)DV;
  auto st = at::cuda::getCurrentCUDAStream();
  if (nc == 0) {
    if (dS_end.has_value()) dS0.copy_(dS_end->view({R, DK, DV}));
    else dS0.zero_();
    return {dU, dSa, dS0};
  }
  if (DK == 128) launch_bwd<128>(a, (int)R, st);
  else launch_bwd<64>(a, (int)R, st);
  return {dU, dSa, dS0};
}

template <typename T>
const T* cptr(const torch::Tensor& t) { return reinterpret_cast<const T*>(t.data_ptr()); }

torch::Tensor gdn_conv_fwd(torch::Tensor x, torch::Tensor w, torch::Tensor prev) {
  TORCH_CHECK(x.is_cuda() && x.is_contiguous() && x.dim() == 2, "x must be a contiguous [T, C] CUDA tensor");
  TORCH_CHECK(w.scalar_type() == x.scalar_type() && w.is_contiguous() && w.size(0) == x.size(1), "w must be [C, W]");
  const int64_t T = x.size(0), C = x.size(1), Wd = w.size(1);
  TORCH_CHECK(Wd >= 1 && Wd <= CONV_MAXW, "conv width must be in [1, 8]");
  TORCH_CHECK(prev.scalar_type() == torch::kInt64 && prev.is_contiguous() && prev.size(0) == T &&
                  prev.size(1) == Wd - 1, "prev must be int64 [T, W-1]");
  auto y = torch::empty({T, C}, x.options().dtype(torch::kFloat32));
  if (T == 0) return y;
  dim3 grid((unsigned)((C + CONV_THREADS - 1) / CONV_THREADS), (unsigned)((T + CONV_ROWS - 1) / CONV_ROWS));
  auto st = at::cuda::getCurrentCUDAStream();
  if (x.scalar_type() == torch::kBFloat16) {
    gdn_conv_fwd_kernel<__nv_bfloat16><<<grid, CONV_THREADS, 0, st>>>(
        cptr<__nv_bfloat16>(x), cptr<__nv_bfloat16>(w), prev.data_ptr<int64_t>(), y.data_ptr<float>(), T, (int)C,
        (int)Wd);
  } else {
    TORCH_CHECK(x.scalar_type() == torch::kFloat32, "x must be bf16 or fp32");
    gdn_conv_fwd_kernel<float><<<grid, CONV_THREADS, 0, st>>>(x.data_ptr<float>(), w.data_ptr<float>(),
                                                             prev.data_ptr<int64_t>(), y.data_ptr<float>(), T,
                                                             (int)C, (int)Wd);
  }
  ART_CUDA_CHECK(cudaGetLastError());
  return y;
}

// Returns [dx (dtype of x), dw fp32].
std::vector<torch::Tensor> gdn_conv_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor prev,
                                        torch::Tensor succ_ptr, torch::Tensor succ_idx, torch::Tensor succ_tap) {
  check_f32(dy, "dy");
  TORCH_CHECK(dy.sizes() == x.sizes() && x.is_contiguous(), "dy shape mismatch");
  const int64_t T = x.size(0), C = x.size(1), Wd = w.size(1);
  TORCH_CHECK(Wd >= 1 && Wd <= CONV_MAXW, "conv width must be in [1, 8]");
  TORCH_CHECK(succ_ptr.scalar_type() == torch::kInt64 && succ_ptr.numel() == T + 1, "succ_ptr must be int64 [T+1]");
  TORCH_CHECK(succ_idx.scalar_type() == torch::kInt64 && succ_tap.scalar_type() == torch::kInt8 &&
                  succ_idx.numel() == succ_tap.numel(), "succ_idx int64 / succ_tap int8 of equal length");
  auto dpre = torch::empty({T, C}, dy.options());
  auto dw = torch::zeros({C, Wd}, dy.options());
  auto dx = torch::empty({T, C}, x.options());
  if (T == 0) return {dx, dw};
  dim3 grid((unsigned)((C + CONV_THREADS - 1) / CONV_THREADS), (unsigned)((T + CONV_ROWS - 1) / CONV_ROWS));
  auto st = at::cuda::getCurrentCUDAStream();
  if (x.scalar_type() == torch::kBFloat16) {
    gdn_conv_dpre_kernel<__nv_bfloat16><<<grid, CONV_THREADS, 0, st>>>(
        dy.data_ptr<float>(), cptr<__nv_bfloat16>(x), cptr<__nv_bfloat16>(w), prev.data_ptr<int64_t>(),
        dpre.data_ptr<float>(), dw.data_ptr<float>(), T, (int)C, (int)Wd);
    gdn_conv_dx_kernel<__nv_bfloat16><<<grid, CONV_THREADS, 0, st>>>(
        dpre.data_ptr<float>(), cptr<__nv_bfloat16>(w), succ_ptr.data_ptr<int64_t>(), succ_idx.data_ptr<int64_t>(),
        succ_tap.data_ptr<int8_t>(), reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), T, (int)C, (int)Wd);
  } else {
    TORCH_CHECK(x.scalar_type() == torch::kFloat32, "x must be bf16 or fp32");
    gdn_conv_dpre_kernel<float><<<grid, CONV_THREADS, 0, st>>>(dy.data_ptr<float>(), x.data_ptr<float>(),
                                                              w.data_ptr<float>(), prev.data_ptr<int64_t>(),
                                                              dpre.data_ptr<float>(), dw.data_ptr<float>(), T,
                                                              (int)C, (int)Wd);
    gdn_conv_dx_kernel<float><<<grid, CONV_THREADS, 0, st>>>(dpre.data_ptr<float>(), w.data_ptr<float>(),
                                                            succ_ptr.data_ptr<int64_t>(), succ_idx.data_ptr<int64_t>(),
                                                            succ_tap.data_ptr<int8_t>(), dx.data_ptr<float>(), T,
                                                            (int)C, (int)Wd);
  }
  ART_CUDA_CHECK(cudaGetLastError());
  return {dx, dw};
}

}  // namespace art
