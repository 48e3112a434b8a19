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

struct GemmArgs {
  int M, N, K2;
  int nk1, nk2;  // k-blocks of the main and the extension product
  __nv_bfloat16* C;
  int64_t ldc;
  const __nv_bfloat16* bias;
  int accumulate_c;
  int* err;
};

__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
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
  const int num_tiles = num_m * num_n;
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
      prefetch_tmap(&tmA);
      prefetch_tmap(&tmB);
      if (p.nk2) {
        prefetch_tmap(&tmA2);
        prefetch_tmap(&tmB2);
      }
      int it = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
        const int m0 = (tile % num_m) * GBM, n0 = (tile / num_m) * GBN;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % GSTAGES;
          const uint32_t ph = (it / GSTAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.err, 1)) break;
          uint8_t* a = smem + s * STAGE_BYTES;
          uint8_t* b = a + A_TILE;
          mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
          if (kb < p.nk1) {
            tma_load_2d(a, &tmA, &full[s], kb * GBK, m0);
            tma_load_2d(b, &tmB, &full[s], kb * GBK, n0);
          } else {
            const int k2 = (kb - p.nk1) * GBK;
            tma_load_2d(a, &tmA2, &full[s], k2, m0);
            tma_load_2d(b, &tmB2, &full[s], k2, n0);
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
          for (int kk = 0; kk < ksteps; ++kk)
            mma_bf16(d, desc_k_sw128(a_addr + kk * 32), desc_k_sw128(b_addr + kk * 32), idesc,
                     (kb > 0 || kk > 0) ? 1u : 0u);
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
      if (!mbar_wait(&acc_full[buf], use & 1, abort_flag, p.err, 4)) break;
      tc_fence_after();
      const int m0 = (tile % num_m) * GBM, n0 = (tile / num_m) * GBN;
      const int row = m0 + q * 32 + lane;
#pragma unroll 1
      for (int c = 0; c < GBN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + buf * GBN + c * 32, r);
        tmem_wait_ld();
        const int col0 = n0 + c * 32;
        if (row < p.M && col0 < p.N) {
          __nv_bfloat16* dst = p.C + (int64_t)row * p.ldc + col0;
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

static torch::Tensor& error_word(int dev) {
  static std::vector<torch::Tensor> words(64);
  if (!words[dev].defined())
    words[dev] = torch::zeros({1}, torch::TensorOptions().dtype(torch::kInt).device(torch::kCUDA, dev));
  return words[dev];
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
  const bool ext = a2.has_value();
  int K2 = 0;
  if (ext) {
    TORCH_CHECK(b2.has_value() && a2->size(0) == M && b2->size(0) == N && a2->size(1) == b2->size(1));
    K2 = a2->size(1);
  }
  if (bias.has_value()) TORCH_CHECK(bias->numel() == N && bias->is_contiguous());
  CUtensorMap ta = make_tmap_2d(a, GBM), tb = make_tmap_2d(b, GBN);
  CUtensorMap ta2 = ext ? make_tmap_2d(*a2, GBM) : ta, tb2 = ext ? make_tmap_2d(*b2, GBN) : tb;
  int dev = a.get_device();
  GemmArgs p;
  p.M = (int)M;
  p.N = (int)N;
  p.K2 = K2;
  p.nk1 = (int)((K + GBK - 1) / GBK);
  p.nk2 = ext ? (K2 + GBK - 1) / GBK : 0;
  p.C = reinterpret_cast<__nv_bfloat16*>(c.data_ptr());
  p.ldc = c.stride(0);
  p.bias = bias.has_value() ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr;
  p.accumulate_c = accumulate ? 1 : 0;
  p.err = error_word(dev).data_ptr<int>();
  static int num_sms = 0;
  if (!num_sms) ART_CUDA_CHECK(cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev));
  const int tiles = (int)(((M + GBM - 1) / GBM) * ((N + GBN - 1) / GBN));
  const int grid = tiles < num_sms ? tiles : num_sms;
  static bool attr = false;
  if (!attr) {
    ART_CUDA_CHECK(cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, GEMM_SMEM));
    attr = true;
  }
  gemm_tc_kernel<<<grid, GEMM_THREADS, GEMM_SMEM, at::cuda::getCurrentCUDAStream()>>>(ta, tb, ta2, tb2, p);
  ART_CUDA_CHECK(cudaGetLastError());
  return c;
}

}  // namespace art
