// tcgen05 GEMM on CTA pairs (cta_group::2) with the fused LoRA K-extension.
//
//   C[M, N] = A[M, K] * B[N, K]^T  +  A2[M, K2] * B2[N, K2]^T  (+ bias[N]) (+ C)
//
// A cluster of two CTAs (on two SMs) computes one 256x256 output tile with
// M=256, N=256 tcgen05.mma instructions issued by one thread of the leader
// CTA: each CTA stages its own 128 rows of A and 128 rows of B (the N half)
// in its shared memory, and its TMEM receives its 128 rows of the
// accumulator.  Per SM and per k-step this reads half the operand bytes of a
// 1-CTA 128x256 tile for the same FLOPs.
//
//   warp 0    TMA producer (each CTA): 7-stage ring of (A 128x64, B 128x64),
//             loads complete on the LEADER's full barrier (plain TMA loads,
//             .cta_group::2 routing of the completion; no multicast);
//   warp 1    TMEM allocation for the pair (512 columns = two 128x256 fp32
//             accumulators per CTA); in the leader, one thread issues the
//             MMAs and commits their completion to both CTAs' barriers;
//   warps 2-5 epilogue (each CTA): tcgen05.ld of its 128 rows, bias /
//             accumulate, bf16, 16-byte stores; then one arrive per warp on
//             the leader's accumulator-empty barrier (remote, via mapa).
//
// Tiles are walked persistently by the clusters in a grouped raster: a group
// holds as many 256-row bands of A as fit in about 48 MB, so the group's A
// stays in L2 while B streams through once per group (B is read once in
// all when A fits).
// Every wait is bounded (tc_common.cuh); TMEM is always freed.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <cudaTypedefs.h>
#include "common.cuh"
#include "tc_common.cuh"

namespace art {
using namespace tc;

namespace {

constexpr int PBM = 256, PBN = 256, PBK = 64, PSTAGES = 7;
constexpr int P_HALF = 128 * PBK * 2;  // 16 KB: 128 rows x 64 bf16
constexpr int P_STAGE = 2 * P_HALF;    // A half + B half, per CTA
constexpr int P_THREADS = 192;
constexpr int P_SMEM = PSTAGES * P_STAGE + 1024 /*align*/ + 256 /*barriers*/;

struct PairArgs {
  int M, N, K2;
  int nk1, nk2;
  __nv_bfloat16* C;
  int64_t ldc;
  const __nv_bfloat16* bias;
  int accumulate_c;
  int group_m;  // pair rows of A per raster group
  int b_mn;     // B of the main product given as [K, N] row-major (MN-major operand)
  int* err;
  // optional pipeline counters (null: off), summed over the leader CTAs:
  // [0] ns the MMA thread waited for operands, [1] ns it waited for a free
  // accumulator, [2] ns from its first wait to its last commit, [3] k-blocks
  // whose operands were not ready at the first probe, [4] k-blocks issued
  unsigned long long* diag;
};

__device__ __forceinline__ int2 pair_tile(int t, int num_m, int num_n, int group_m) {
  const int group = group_m * num_n;
  const int g = t / group;
  const int first_m = g * group_m;
  const int gm = min(num_m - first_m, group_m);
  const int r = t - g * group;
  return make_int2((first_m + r % gm) * PBM, (r / gm) * PBN);
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(P_THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2,
                     const PairArgs p) {
  extern __shared__ uint8_t smem_raw[];
  // same offset in both CTAs: the MMA descriptors and mapa rely on it
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + PSTAGES * P_STAGE);
  uint64_t* empty = full + PSTAGES;
  uint64_t* acc_full = empty + PSTAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int num_m = (p.M + PBM - 1) / PBM;
  const int num_n = (p.N + PBN - 1) / PBN;
  const int num_tiles = num_m * num_n;
  const int nk = p.nk1 + p.nk2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < PSTAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 8);  // one arrive per epilogue warp of both CTAs
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, 512);
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&tmA);
      prefetch_tmap(&tmB);
      if (p.nk2) {
        prefetch_tmap(&tmA2);
        prefetch_tmap(&tmB2);
      }
      const uint32_t full_leader = mapa_shared(smem_addr(full), 0);
      int it = 0;
      for (int t = pair; t < num_tiles && !*abort_flag; t += npairs) {
        const int2 c = pair_tile(t, num_m, num_n, p.group_m);
        const int am = c.x + (int)rank * 128, bn = c.y + (int)rank * 128;
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % PSTAGES;
          const uint32_t ph = (it / PSTAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.err, 21)) {
            ok = false;
            break;
          }
          uint8_t* a = smem + s * P_STAGE;
          uint8_t* b = a + P_HALF;
          const uint32_t fb = full_leader + s * 8;
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * P_STAGE);  // both CTAs' bytes
          if (kb < p.nk1) {
            tma_load_2d_pair(a, &tmA, fb, kb * PBK, am);
            if (p.b_mn) {  // two 64-column boxes of the [K, N] matrix: 64 K rows each
              tma_load_2d_pair(b, &tmB, fb, bn, kb * PBK);
              tma_load_2d_pair(b + P_HALF / 2, &tmB, fb, bn + 64, kb * PBK);
            } else {
              tma_load_2d_pair(b, &tmB, fb, kb * PBK, bn);
            }
          } else {
            const int k2 = (kb - p.nk1) * PBK;
            tma_load_2d_pair(a, &tmA2, fb, k2, am);
            tma_load_2d_pair(b, &tmB2, fb, k2, bn);
          }
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA (leader)
    if (leader && lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(PBM, PBN);
      unsigned long long d_full = 0, d_acc = 0, d_miss = 0, d_blocks = 0;
      const uint64_t t_start = p.diag ? gtimer() : 0;
      int it = 0, tl = 0;
      for (int t = pair; t < num_tiles && !*abort_flag; t += npairs, ++tl) {
        const int buf = tl & 1;
        const uint32_t use = (uint32_t)(tl >> 1);
        const uint64_t ta = p.diag ? gtimer() : 0;
        if (!mbar_wait(&acc_empty[buf], (use & 1) ^ 1, abort_flag, p.err, 22)) break;
        if (p.diag) d_acc += gtimer() - ta;
        tc_fence_after();
        const uint32_t d = tmem + buf * PBN;
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % PSTAGES;
          const uint32_t ph = (it / PSTAGES) & 1;
          if (p.diag) {
            ++d_blocks;
            if (!mbar_try_wait(&full[s], ph)) {
              ++d_miss;
              const uint64_t tf = gtimer();
              if (!mbar_wait(&full[s], ph, abort_flag, p.err, 23)) {
                ok = false;
                break;
              }
              d_full += gtimer() - tf;
            }
          } else if (!mbar_wait(&full[s], ph, abort_flag, p.err, 23)) {
            ok = false;
            break;
          }
          // operands arrive through the async proxy (TMA) and the barrier
          // orders them for the MMA: no thread-sync fence per k-block
          const uint32_t a_addr = smem_addr(smem + s * P_STAGE);
          const uint64_t da = desc_k_sw128(a_addr), db = desc_k_sw128(a_addr + P_HALF);
          if (kb < p.nk1 && p.b_mn) {
            // MN-major B: 16 K rows of 128 B per step (+2048 B), 64-column chunks 8 KB apart
            const uint64_t dbm = desc_mn_sw128(a_addr + P_HALF, P_HALF / 2);
#pragma unroll
            for (int kk = 0; kk < PBK / 16; ++kk)
              mma_bf16_pair(d, da + 2 * kk, dbm + 128 * kk, idesc | (1u << 16), (kb > 0 || kk > 0) ? 1u : 0u);
          } else if (kb < p.nk1) {
#pragma unroll
            for (int kk = 0; kk < PBK / 16; ++kk)  // +32 bytes per K=16 step (descriptor units of 16 B)
              mma_bf16_pair(d, da + 2 * kk, db + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          } else {
            const int rem = p.K2 - (kb - p.nk1) * PBK;
            const int ksteps = min(PBK / 16, (rem + 15) / 16);
            for (int kk = 0; kk < ksteps; ++kk)
              mma_bf16_pair(d, da + 2 * kk, db + 2 * kk, idesc, 1u);
          }
          mma_commit_pair_both(&empty[s], 0x3);
        }
        if (!ok) break;
        mma_commit_pair_both(&acc_full[buf], 0x3);
      }
      if (p.diag) {
        atomicAdd(p.diag + 0, d_full);
        atomicAdd(p.diag + 1, d_acc);
        atomicAdd(p.diag + 2, (unsigned long long)(gtimer() - t_start));
        atomicAdd(p.diag + 3, d_miss);
        atomicAdd(p.diag + 4, d_blocks);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quadrant of this warp
    const uint32_t acce_leader = mapa_shared(smem_addr(acc_empty), 0);
    int tl = 0;
    for (int t = pair; t < num_tiles; t += npairs, ++tl) {
      const int buf = tl & 1;
      const uint32_t use = (uint32_t)(tl >> 1);
      if (!mbar_wait_warp(&acc_full[buf], use & 1, abort_flag, p.err, 24)) break;
      tc_fence_after();
      const int2 c = pair_tile(t, num_m, num_n, p.group_m);
      const int row = c.x + (int)rank * 128 + q * 32 + lane;
#pragma unroll 1
      for (int cc = 0; cc < PBN / 32; cc += 2) {
        uint32_t r2[2][32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + buf * PBN + cc * 32, r2[0]);
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + buf * PBN + (cc + 1) * 32, r2[1]);
        tmem_wait_ld();
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int col0 = c.y + (cc + h) * 32;
          if (row < p.M && col0 < p.N) {
            __nv_bfloat16* dst = p.C + (int64_t)row * p.ldc + col0;
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r2[h][j]);
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
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acce_leader + buf * 8);
    }
  }
  tc_fence_before();
  cluster_sync();  // no MMA, TMEM read or remote arrive of either CTA is still pending
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

}  // namespace

// out = a @ b^T (+ a2 @ b2^T) (+ bias) (+ out if accumulate), on CTA pairs;
// with b_transposed, b is given as [K, N] (out = a @ b): the frozen weight of
// a linear layer in its stored layout for the input-gradient GEMM.
torch::Tensor gemm_pair(torch::Tensor a, torch::Tensor b, c10::optional<torch::Tensor> a2,
                        c10::optional<torch::Tensor> b2, c10::optional<torch::Tensor> bias,
                        c10::optional<torch::Tensor> out, bool accumulate, c10::optional<torch::Tensor> diag,
                        bool b_transposed) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda());
  const int64_t M = a.size(0), K = a.size(1), N = b_transposed ? b.size(1) : b.size(0);
  TORCH_CHECK((b_transposed ? b.size(0) : b.size(1)) == K, "inner dimensions differ");
  if (b_transposed) TORCH_CHECK(N % 128 == 0, "transposed B: N must be a multiple of 128");
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
  if (a2.has_value())
    TORCH_CHECK(b2.has_value() && a2->size(0) == M && b2->size(0) == N && a2->size(1) == b2->size(1));
  if (bias.has_value()) TORCH_CHECK(bias->numel() == N && bias->is_contiguous());
  const CUtensorMap ta = make_tmap_bf16(a, 128), tb = make_tmap_bf16(b, b_transposed ? 64 : 128);
  const CUtensorMap ta2 = a2.has_value() ? make_tmap_bf16(*a2, 128) : ta;
  const CUtensorMap tb2 = a2.has_value() ? make_tmap_bf16(*b2, 128) : tb;
  PairArgs p;
  p.M = (int)M;
  p.N = (int)N;
  p.K2 = a2.has_value() ? (int)a2->size(1) : 0;
  p.nk1 = (int)((K + PBK - 1) / PBK);
  p.nk2 = a2.has_value() ? (p.K2 + PBK - 1) / PBK : 0;
  p.C = reinterpret_cast<__nv_bfloat16*>(c.data_ptr());
  p.ldc = c.stride(0);
  p.bias = bias.has_value() ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr;
  p.accumulate_c = accumulate ? 1 : 0;
  p.b_mn = b_transposed ? 1 : 0;
  p.diag = nullptr;
  if (diag.has_value()) {
    TORCH_CHECK(diag->is_cuda() && diag->scalar_type() == torch::kInt64 && diag->numel() >= 5, "diag: int64[5]");
    p.diag = reinterpret_cast<unsigned long long*>(diag->data_ptr<int64_t>());
  }
  {
    const int64_t num_m = (M + PBM - 1) / PBM;
    const int64_t band = (int64_t)PBM * K * 2;  // bytes of one 256-row band of A
    int64_t g = ((int64_t)48 << 20) / (band > 0 ? band : 1);
    p.group_m = (int)std::max<int64_t>(1, std::min<int64_t>(g, num_m));
  }
  const int dev = a.get_device();
  p.err = tc_error_ptr(dev);
  static int max_pairs[64] = {0};
  if (!max_pairs[dev]) {
    ART_CUDA_CHECK(cudaFuncSetAttribute(gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(P_THREADS, 1, 1);
    cfg.dynamicSmemBytes = P_SMEM;  // cluster shape comes from __cluster_dims__
    int n = 0;
    ART_CUDA_CHECK(cudaOccupancyMaxActiveClusters(&n, gemm_pair_kernel, &cfg));
    TORCH_CHECK(n > 0, "no CTA pair of the GEMM fits on this device");
    max_pairs[dev] = n;
  }
  const int tiles = (int)(((M + PBM - 1) / PBM) * ((N + PBN - 1) / PBN));
  const int pairs = tiles < max_pairs[dev] ? tiles : max_pairs[dev];
  gemm_pair_kernel<<<2 * pairs, P_THREADS, P_SMEM, at::cuda::getCurrentCUDAStream()>>>(ta, tb, ta2, tb2, p);
  ART_CUDA_CHECK(cudaGetLastError());
  return c;
}

}  // namespace art
