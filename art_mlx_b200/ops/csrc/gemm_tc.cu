// tcgen05 / TMEM GEMM for sm_100a with a fused low-rank (LoRA) K-extension.
//
//   C[M, N] = A[M, K] * B[N, K]^T  +  A2[M, K2] * B2[N, K2]^T  (+ bias[N]) (+ C)
//
// All operands bf16 and K-major (row-major activations, nn.Linear weights);
// fp32 accumulation in tensor memory; bf16 output.  For a LoRA projection the
// extension operands are  A2 = x A^T  (rank r, tiny) and  B2 = scale * B,
// so the adapter costs one more k-step in the same accumulator instead of a
// second pass over the output.
//
// Structure (one CTA per SM, persistent over 128x256 output tiles, M-fastest
// so consecutive CTAs share a weight tile through L2):
//   warp 0      TMA producer: 4-stage ring of (A 128x64, B 256x64) tiles,
//               128-byte swizzle, completion on per-stage mbarriers;
//   warp 1      allocates 512 TMEM columns (two 128x256 fp32 accumulators)
//               and issues tcgen05.mma (M=128, N=256, K=16) from one thread;
//               tcgen05.commit releases smem stages and publishes accumulators;
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns per warp quadrant,
//               bias / accumulate, bf16 convert, 16-byte global stores; the
//               accumulator is released back to the MMA warp (double buffer).
// Every mbarrier wait is bounded (see tc_common.cuh); TMEM is always freed.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <cudaTypedefs.h>
#include "common.cuh"
#include "tc_common.cuh"

namespace art {
using namespace tc;

constexpr int GBM = 128, GBN = 256, GBK = 64, GSTAGES = 4;
constexpr int A_TILE = GBM * GBK * 2;  // 16 KB
constexpr int B_TILE = GBN * GBK * 2;  // 32 KB
constexpr int STAGE_BYTES = A_TILE + B_TILE;
constexpr int GEMM_THREADS = 192;
constexpr int GEMM_SMEM = GSTAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;

constexpr int MAX_SRC = 8;

struct GemmArgs {
  int M, N, K2;
  int nk1, nk2;  // k-blocks of the main and the extension product
  __nv_bfloat16* C;
  int64_t ldc;
  const __nv_bfloat16* bias;
  int accumulate_c;
  int* err;
  // multi-source A (all-gather fused into the load): rows [s*a_src_rows,
  // (s+1)*a_src_rows) of A are read through tensor map s (0 = single source)
  int a_src_rows;
  // scattered output (reduce-scatter fused into the epilogue): rows
  // [r*c_dst_rows, (r+1)*c_dst_rows) go to c_bases[r] at row offset
  // c_slot*c_dst_rows (0 = plain C)
  int c_dst_rows;
  int c_slot;
  long long c_bases[MAX_SRC];
  // grouped mode (MoE experts): tile list of (m0, n0, first B row, row end);
  // B and B2 are the experts' matrices stacked along rows, A rows of tile t
  // are valid up to row end (the next expert's rows are computed, not stored)
  const int4* tiles;
  int num_tiles;
  // B of the main product given transposed, as [K, N] row-major (MN-major
  // operand: four 64-column TMA boxes per k-block, read with an MN-major
  // descriptor); the tile's B row is then the first K row of its matrix
  int b_mn;
  int kmain;  // K of the main product (transposed-B tiles: B2 row = (brow / K) * N + n0)
};

struct TmapSet {
  CUtensorMap m[MAX_SRC];
};

__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ TmapSet tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2,
                   const GemmArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + GSTAGES * STAGE_BYTES);
  uint64_t* empty = full + GSTAGES;
  uint64_t* acc_full = empty + GSTAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (p.M + GBM - 1) / GBM;
  const int num_n = (p.N + GBN - 1) / GBN;
  const int num_tiles = p.tiles ? p.num_tiles : num_m * num_n;
  // tile -> (m0, n0, row of B, end of valid A rows)
  auto coords = [&](int tile) -> int4 {
    if (p.tiles) return __ldg(p.tiles + tile);
    const int m0 = (tile % num_m) * GBM, n0 = (tile / num_m) * GBN;
    return make_int4(m0, n0, n0, p.M);
  };
  const int nk = p.nk1 + p.nk2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < GSTAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const int nsrc = p.a_src_rows ? (p.M + p.a_src_rows - 1) / p.a_src_rows : 1;
      for (int q = 0; q < nsrc && q < MAX_SRC; ++q) prefetch_tmap(&tmA.m[q]);
      prefetch_tmap(&tmB);
      if (p.nk2) {
        prefetch_tmap(&tmA2);
        prefetch_tmap(&tmB2);
      }
      int it = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
        const int4 tc4 = coords(tile);
        const int m0 = tc4.x, n0 = tc4.y, brow = tc4.z;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % GSTAGES;
          const uint32_t ph = (it / GSTAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.err, 1)) break;
          uint8_t* a = smem + s * STAGE_BYTES;
          uint8_t* b = a + A_TILE;
          mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
          if (kb < p.nk1) {
            if (p.a_src_rows) {
              const int q = m0 / p.a_src_rows;
              tma_load_2d(a, &tmA.m[q], &full[s], kb * GBK, m0 - q * p.a_src_rows);
            } else {
              tma_load_2d(a, &tmA.m[0], &full[s], kb * GBK, m0);
            }
            if (p.b_mn) {
#pragma unroll
              for (int j = 0; j < GBN / 64; ++j)
                tma_load_2d(b + j * (GBK * 128), &tmB, &full[s], n0 + 64 * j, brow + kb * GBK);
            } else {
              tma_load_2d(b, &tmB, &full[s], kb * GBK, brow);
            }
          } else {
            const int k2 = (kb - p.nk1) * GBK;
            const int b2row = p.b_mn ? (brow / p.kmain) * p.N + n0 : brow;
            tma_load_2d(a, &tmA2, &full[s], k2, m0);
            tma_load_2d(b, &tmB2, &full[s], k2, b2row);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(GBM, GBN);
      int it = 0, t = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x, ++t) {
        const int buf = t & 1;
        const uint32_t use = (uint32_t)(t >> 1);
        if (!mbar_wait(&acc_empty[buf], (use & 1) ^ 1, abort_flag, p.err, 2)) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * GBN;
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % GSTAGES;
          const uint32_t ph = (it / GSTAGES) & 1;
          if (!mbar_wait(&full[s], ph, abort_flag, p.err, 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_addr(smem + s * STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_TILE;
          int ksteps = GBK / 16;
          if (kb >= p.nk1) {
            const int rem = p.K2 - (kb - p.nk1) * GBK;
            ksteps = min(ksteps, (rem + 15) / 16);
          }
          const bool bmn = p.b_mn && kb < p.nk1;
          for (int kk = 0; kk < ksteps; ++kk)
            mma_bf16(d, desc_k_sw128(a_addr + kk * 32),
                     bmn ? desc_mn_sw128(b_addr + kk * 2048, GBK * 128) : desc_k_sw128(b_addr + kk * 32),
                     bmn ? (idesc | (1u << 16)) : idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&empty[s]);
        }
        if (!ok) break;
        mma_commit(&acc_full[buf]);
      }
    }
  } else {
    // epilogue warps 2..5 -> TMEM lane quadrants 2,3,0,1
    const int q = warp & 3;
    int t = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++t) {
      const int buf = t & 1;
      const uint32_t use = (uint32_t)(t >> 1);
      if (!mbar_wait_warp(&acc_full[buf], use & 1, abort_flag, p.err, 4)) break;
      tc_fence_after();
      const int4 tc4 = coords(tile);
      const int m0 = tc4.x, n0 = tc4.y, row_end = tc4.w;
      const int row = m0 + q * 32 + lane;
#pragma unroll 1
      for (int c = 0; c < GBN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + buf * GBN + c * 32, r);
        tmem_wait_ld();
        const int col0 = n0 + c * 32;
        if (row < row_end && col0 < p.N) {
          __nv_bfloat16* dst;
          if (p.c_dst_rows) {
            const int rr = row / p.c_dst_rows;
            dst = reinterpret_cast<__nv_bfloat16*>(p.c_bases[rr]) +
                  ((int64_t)p.c_slot * p.c_dst_rows + (row - rr * p.c_dst_rows)) * p.ldc + col0;
          } else {
            dst = p.C + (int64_t)row * p.ldc + col0;
          }
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
          if (p.bias) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
              uint4 bv = *reinterpret_cast<const uint4*>(p.bias + col0 + j);
              const __nv_bfloat16* be = reinterpret_cast<const __nv_bfloat16*>(&bv);
#pragma unroll
              for (int e = 0; e < 8; ++e) v[j + e] += bf2f(be[e]);
            }
          }
          if (p.accumulate_c) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
              uint4 cv = *reinterpret_cast<const uint4*>(dst + j);
              const __nv_bfloat16* ce = reinterpret_cast<const __nv_bfloat16*>(&cv);
#pragma unroll
              for (int e = 0; e < 8; ++e) v[j + e] += bf2f(ce[e]);
            }
          }
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            uint4 o;
            o.x = pack_bf16x2(v[j + 0], v[j + 1]);
            o.y = pack_bf16x2(v[j + 2], v[j + 3]);
            o.z = pack_bf16x2(v[j + 4], v[j + 5]);
            o.w = pack_bf16x2(v[j + 6], v[j + 7]);
            *reinterpret_cast<uint4*>(dst + j) = o;
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------- host side
// The driver entry point is resolved at run time (through the runtime API) so
// the extension has no link-time dependency on libcuda and imports on hosts
// without a GPU driver.
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    ART_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && ptr, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

static CUtensorMap make_tmap_2d(const torch::Tensor& t, int box_rows) {
  TORCH_CHECK(t.scalar_type() == at::kBFloat16 && t.dim() == 2 && t.stride(1) == 1, "bf16 row-major 2-D tensor");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(t.data_ptr()) % 16) == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((t.stride(0) * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)t.size(1), (cuuint64_t)t.size(0)};
  cuuint64_t strides[1] = {(cuuint64_t)(t.stride(0) * 2)};
  cuuint32_t box[2] = {(cuuint32_t)GBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, t.data_ptr(), dims, strides, box,
                                      estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
  return m;
}

CUtensorMap make_tmap_bf16(const at::Tensor& t, int box_rows) { return make_tmap_2d(t, box_rows); }

CUtensorMap make_tmap_f32_32(const at::Tensor& t) {
  TORCH_CHECK(t.scalar_type() == at::kFloat && t.dim() == 2 && t.stride(1) == 1, "fp32 row-major 2-D tensor");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(t.data_ptr()) % 16) == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((t.stride(0) * 4) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)t.size(1), (cuuint64_t)t.size(0)};
  cuuint64_t strides[1] = {(cuuint64_t)(t.stride(0) * 4)};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, t.data_ptr(), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
  return m;
}

static torch::Tensor& error_word(int dev) {
  static std::vector<torch::Tensor> words(64);
  if (!words[dev].defined())
    words[dev] = torch::zeros({1}, torch::TensorOptions().dtype(torch::kInt).device(torch::kCUDA, dev));
  return words[dev];
}

int* tc_error_ptr(int dev) { return error_word(dev).data_ptr<int>(); }

// The device error word itself (int32 [1] on the current device), so a
// caller can fold it into a step's status read without a separate sync.
torch::Tensor tc_error_word() {
  int dev = 0;
  ART_CUDA_CHECK(cudaGetDevice(&dev));
  return error_word(dev);
}

// Returns and clears the device error word of the tensor-core kernels
// (0 = ok; 1..4 = which pipeline wait timed out).
int64_t tc_error_code() {
  int dev = 0;
  ART_CUDA_CHECK(cudaGetDevice(&dev));
  auto& w = error_word(dev);
  int64_t v = w.item<int>();
  if (v) w.zero_();
  return v;
}

static void launch_gemm(const TmapSet& ta, const CUtensorMap& tb, const CUtensorMap& ta2, const CUtensorMap& tb2,
                        GemmArgs& p, int dev) {
  p.err = error_word(dev).data_ptr<int>();
  static int num_sms = 0;
  if (!num_sms) ART_CUDA_CHECK(cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev));
  const int tiles = p.tiles ? p.num_tiles : ((p.M + GBM - 1) / GBM) * ((p.N + GBN - 1) / GBN);
  const int grid = tiles < num_sms ? tiles : num_sms;
  static bool attr = false;
  if (!attr) {
    ART_CUDA_CHECK(cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, GEMM_SMEM));
    attr = true;
  }
  if (grid > 0)
    gemm_tc_kernel<<<grid, GEMM_THREADS, GEMM_SMEM, at::cuda::getCurrentCUDAStream()>>>(ta, tb, ta2, tb2, p);
  ART_CUDA_CHECK(cudaGetLastError());
}

static void fill_common(GemmArgs& p, int64_t M, int64_t K, int64_t N, const c10::optional<torch::Tensor>& a2,
                        const c10::optional<torch::Tensor>& bias, bool accumulate) {
  p.M = (int)M;
  p.N = (int)N;
  p.K2 = a2.has_value() ? (int)a2->size(1) : 0;
  p.nk1 = (int)((K + GBK - 1) / GBK);
  p.nk2 = a2.has_value() ? (p.K2 + GBK - 1) / GBK : 0;
  p.bias = bias.has_value() ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr;
  p.accumulate_c = accumulate ? 1 : 0;
  p.a_src_rows = 0;
  p.c_dst_rows = 0;
  p.c_slot = 0;
  for (int i = 0; i < MAX_SRC; ++i) p.c_bases[i] = 0;
  p.tiles = nullptr;
  p.num_tiles = 0;
  p.b_mn = 0;
  p.kmain = (int)K;
}

// out = a @ b^T (+ a2 @ b2^T) (+ bias) (+ out if accumulate)
torch::Tensor gemm_tc(torch::Tensor a, torch::Tensor b, c10::optional<torch::Tensor> a2,
                      c10::optional<torch::Tensor> b2, c10::optional<torch::Tensor> bias,
                      c10::optional<torch::Tensor> out, bool accumulate) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda());
  const int64_t M = a.size(0), K = a.size(1), N = b.size(0);
  TORCH_CHECK(b.size(1) == K, "inner dimensions differ");
  TORCH_CHECK(N % 32 == 0, "N must be a multiple of 32");
  torch::Tensor c;
  if (out.has_value()) {
    c = *out;
    TORCH_CHECK(c.size(0) == M && c.size(1) == N && c.stride(1) == 1 && c.stride(0) % 8 == 0);
  } else {
    TORCH_CHECK(!accumulate);
    c = torch::empty({M, N}, a.options());
  }
  if (M == 0) return c;
  if (a2.has_value()) TORCH_CHECK(b2.has_value() && a2->size(0) == M && b2->size(0) == N && a2->size(1) == b2->size(1));
  if (bias.has_value()) TORCH_CHECK(bias->numel() == N && bias->is_contiguous());
  TmapSet ta;
  ta.m[0] = make_tmap_2d(a, GBM);
  CUtensorMap tb = make_tmap_2d(b, GBN);
  CUtensorMap ta2 = a2.has_value() ? make_tmap_2d(*a2, GBM) : ta.m[0];
  CUtensorMap tb2 = a2.has_value() ? make_tmap_2d(*b2, GBN) : tb;
  GemmArgs p;
  fill_common(p, M, K, N, a2, bias, accumulate);
  p.C = reinterpret_cast<__nv_bfloat16*>(c.data_ptr());
  p.ldc = c.stride(0);
  launch_gemm(ta, tb, ta2, tb2, p, a.get_device());
  return c;
}

// Grouped GEMM for MoE experts: rows [offs[e], offs[e+1]) of x belong to
// expert e;  out[rows_e] = x[rows_e] W_e^T (+ a2[rows_e] B2_e^T), W = w viewed
// as [E*N, K] (expert-major), or, with w_transposed, w = the stacked W_e^T as
// [E*K, N]; B2 = b2 as [E*N, K2].  offs are host ints (the routing plan is
// built on the host).  N must be a multiple of 32 (of 64 when transposed).
torch::Tensor gemm_tc_grouped(torch::Tensor x, torch::Tensor w, std::vector<int64_t> offs, int64_t N,
                              c10::optional<torch::Tensor> a2, c10::optional<torch::Tensor> b2,
                              bool w_transposed) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && x.dim() == 2 && w.dim() == 2);
  const int64_t M = x.size(0), K = x.size(1);
  const int64_t E = (int64_t)offs.size() - 1;
  TORCH_CHECK(E >= 1 && offs[0] == 0 && offs[E] == M, "offsets must span the rows");
  if (w_transposed) {
    TORCH_CHECK(w.size(0) == E * K && w.size(1) == N && N % 64 == 0, "w must be [E*K, N]");
  } else {
    TORCH_CHECK(w.size(0) == E * N && w.size(1) == K && N % 32 == 0, "w must be [E*N, K]");
  }
  if (a2.has_value())
    TORCH_CHECK(b2.has_value() && a2->size(0) == M && b2->size(0) == E * N && a2->size(1) == b2->size(1));
  auto c = torch::empty({M, N}, x.options());
  if (M == 0) return c;
  std::vector<int32_t> tab;
  for (int64_t e = 0; e < E; ++e) {
    TORCH_CHECK(offs[e + 1] >= offs[e], "offsets must be non-decreasing");
    for (int64_t n0 = 0; n0 < N; n0 += GBN)
      for (int64_t m0 = offs[e]; m0 < offs[e + 1]; m0 += GBM) {
        tab.push_back((int32_t)m0);
        tab.push_back((int32_t)n0);
        tab.push_back((int32_t)(w_transposed ? e * K : e * N + n0));
        tab.push_back((int32_t)offs[e + 1]);
      }
  }
  const int ntiles = (int)(tab.size() / 4);
  if (ntiles == 0) return c;
  auto tiles = torch::from_blob(tab.data(), {(int64_t)tab.size()}, torch::kInt32).pin_memory().to(x.device(), true);
  TmapSet ta;
  ta.m[0] = make_tmap_2d(x, GBM);
  for (int q = 1; q < MAX_SRC; ++q) ta.m[q] = ta.m[0];
  CUtensorMap tb = make_tmap_2d(w, w_transposed ? GBK : GBN);
  CUtensorMap ta2 = a2.has_value() ? make_tmap_2d(*a2, GBM) : ta.m[0];
  CUtensorMap tb2 = a2.has_value() ? make_tmap_2d(*b2, GBN) : tb;
  GemmArgs p;
  fill_common(p, M, K, N, a2, c10::nullopt, false);
  p.C = reinterpret_cast<__nv_bfloat16*>(c.data_ptr());
  p.ldc = c.stride(0);
  p.b_mn = w_transposed ? 1 : 0;
  p.tiles = reinterpret_cast<const int4*>(tiles.data_ptr<int>());
  p.num_tiles = ntiles;
  launch_gemm(ta, tb, ta2, tb2, p, x.get_device());
  return c;
}

// All-gather fused into the GEMM: A = concat_s(shard_s) where shard s is a
// [rows, K] bf16 matrix at address a_ptrs[s] (peer memory allowed: plain TMA
// loads, no multicast).  rows must be a multiple of 128.
torch::Tensor gemm_tc_ag(std::vector<int64_t> a_ptrs, int64_t rows, int64_t K, int64_t lda, torch::Tensor b,
                         c10::optional<torch::Tensor> a2, c10::optional<torch::Tensor> b2,
                         c10::optional<torch::Tensor> bias) {
  const int nsrc = (int)a_ptrs.size();
  TORCH_CHECK(nsrc >= 1 && nsrc <= MAX_SRC && rows % GBM == 0);
  const int64_t M = rows * nsrc, N = b.size(0);
  TORCH_CHECK(b.size(1) == K && N % 32 == 0);
  auto opts = b.options();
  auto c = torch::empty({M, N}, opts);
  TmapSet ta;
  for (int q = 0; q < nsrc; ++q) {
    auto view = torch::from_blob(reinterpret_cast<void*>(a_ptrs[q]), {rows, K}, {lda, 1}, opts);
    ta.m[q] = make_tmap_2d(view, GBM);
  }
  for (int q = nsrc; q < MAX_SRC; ++q) ta.m[q] = ta.m[0];
  CUtensorMap tb = make_tmap_2d(b, GBN);
  if (a2.has_value()) TORCH_CHECK(b2.has_value() && a2->size(0) == M && b2->size(0) == N);
  CUtensorMap ta2 = a2.has_value() ? make_tmap_2d(*a2, GBM) : ta.m[0];
  CUtensorMap tb2 = a2.has_value() ? make_tmap_2d(*b2, GBN) : tb;
  GemmArgs p;
  fill_common(p, M, K, N, a2, bias, false);
  p.a_src_rows = (int)rows;
  p.C = reinterpret_cast<__nv_bfloat16*>(c.data_ptr());
  p.ldc = c.stride(0);
  launch_gemm(ta, tb, ta2, tb2, p, b.get_device());
  return c;
}

// Reduce-scatter fused into the epilogue: C rows [r*rows, (r+1)*rows) are
// stored into the staging buffer of rank r (c_ptrs[r], peer memory) at slot
// `slot`: staging_r[slot*rows + i, :].  The owner sums the slots afterwards.
void gemm_tc_rs(torch::Tensor a, torch::Tensor b, c10::optional<torch::Tensor> a2, c10::optional<torch::Tensor> b2,
                std::vector<int64_t> c_ptrs, int64_t rows, int64_t ldc, int64_t slot) {
  const int64_t M = a.size(0), K = a.size(1), N = b.size(0);
  const int ndst = (int)c_ptrs.size();
  TORCH_CHECK(ndst >= 1 && ndst <= MAX_SRC && rows * ndst == M && N % 32 == 0 && ldc % 8 == 0);
  TmapSet ta;
  ta.m[0] = make_tmap_2d(a, GBM);
  for (int q = 1; q < MAX_SRC; ++q) ta.m[q] = ta.m[0];
  CUtensorMap tb = make_tmap_2d(b, GBN);
  if (a2.has_value()) TORCH_CHECK(b2.has_value() && a2->size(0) == M && b2->size(0) == N);
  CUtensorMap ta2 = a2.has_value() ? make_tmap_2d(*a2, GBM) : ta.m[0];
  CUtensorMap tb2 = a2.has_value() ? make_tmap_2d(*b2, GBN) : tb;
  GemmArgs p;
  fill_common(p, M, K, N, a2, c10::nullopt, false);
  p.C = nullptr;
  p.ldc = ldc;
  p.c_dst_rows = (int)rows;
  p.c_slot = (int)slot;
  for (int q = 0; q < ndst; ++q) p.c_bases[q] = c_ptrs[q];
  launch_gemm(ta, tb, ta2, tb2, p, a.get_device());
}

// Owner side of the fused reduce-scatter: out[i] = sum_s staging[s*rows + i] (+ residual).
__global__ void slot_sum_kernel(const __nv_bfloat16* __restrict__ staging, int nslots, int64_t rows, int N,
                                const __nv_bfloat16* __restrict__ res, __nv_bfloat16* __restrict__ out) {
  const int64_t nv = rows * (N / 8);
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nv; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = v / (N / 8);
    const int c = (v % (N / 8)) * 8;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int s = 0; s < nslots; ++s) {
      uint4 x = *reinterpret_cast<const uint4*>(staging + ((int64_t)s * rows + i) * N + c);
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&x);
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] += bf2f(e[k]);
    }
    if (res) {
      uint4 x = *reinterpret_cast<const uint4*>(res + i * N + c);
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&x);
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] += bf2f(e[k]);
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + i * N + c) = o;
  }
}

torch::Tensor slot_sum(torch::Tensor staging, int64_t nslots, int64_t rows, c10::optional<torch::Tensor> res) {
  const int N = staging.size(1);
  TORCH_CHECK(staging.is_contiguous() && N % 8 == 0 && staging.size(0) >= nslots * rows);
  auto out = torch::empty({rows, N}, staging.options());
  int64_t blocks = (rows * N / 8 + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (rows > 0)
    slot_sum_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(staging.data_ptr()), (int)nslots, rows, N,
        res.has_value() ? reinterpret_cast<const __nv_bfloat16*>(res->data_ptr()) : nullptr,
        reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  ART_CUDA_CHECK(cudaGetLastError());
  return out;
}

}  // namespace art
