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
//   warp 0    TMA producer (each CTA): 6-stage ring of (A 128x64, B 128x64),
//             loads complete on the LEADER's full barrier (plain TMA loads,
//             .cta_group::2 routing of the completion; no multicast);
//   warp 1    TMEM allocation for the pair (512 columns = two 128x256 fp32
//             accumulators per CTA); in the leader, one thread issues the
//             MMAs and commits their completion to both CTAs' barriers;
//   warps 2-5 epilogue (each CTA): tcgen05.ld of its 128 rows, bias, bf16
//             into a per-warp shared-memory block (16-byte units XOR-swizzled
//             by row), read back so that each store instruction writes 4 rows
//             x 128 contiguous bytes (whole L2 lines, no partial sectors);
//             then one arrive per warp on the leader's accumulator-empty
//             barrier (remote, via mapa).  They wait for an accumulator with
//             a sleeping poll: two of them share SM sub-partitions with the
//             producer and MMA warps.
//
// Tiles are walked persistently by the clusters in a grouped raster: a group
// holds as many 256-row bands of A as fit in about 48 MB, so the group's A
// stays in L2 while B streams through once per group (B is read once in
// all when A fits).
// Every wait is bounded (tc_common.cuh); TMEM is always freed.
#include <cmath>
#include <cstdlib>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <cudaTypedefs.h>
#include "common.cuh"
#include "tc_common.cuh"

namespace art {
using namespace tc;

namespace {

constexpr int PBM = 256, PBN = 256, PBK = 64;  // PBN: N of one MMA
constexpr int P_HALF = 128 * PBK * 2;  // 16 KB: 128 rows x 64 bf16
constexpr int P_THREADS = 192;
constexpr int P_STG_WARP = 32 * 128;   // epilogue staging per warp: 32 rows x 64 bf16 (128 B a row)

// Tile shapes of the pair kernel.  TN = 256: one N=256 MMA per k-step, two
// accumulator buffers (the epilogue of tile t overlaps the mainloop of t+1).
// TN = 512: two N=256 MMAs per k-step reuse each staged A tile, so a k-block
// stages 48 KB per CTA for twice the MMAs (shared memory carries the TMA
// writes and the MMA operand reads at once; the wide tile lowers the former
// by a quarter per FLOP), at the price of one accumulator buffer.
template <int TN>
struct PTile {
  static constexpr int NB = TN / 256;                 // N=256 MMAs per k-step
  static constexpr int NBUF = TN == 256 ? 2 : 1;      // accumulator buffers in the 512 TMEM columns
  static constexpr int STAGES = TN == 256 ? 6 : 4;
  static constexpr int STAGE = P_HALF * (1 + NB);     // A half + this CTA's B halves
  static constexpr int SMEM = STAGES * STAGE + 1024 /*align*/ + 256 /*barriers*/ + 4 * P_STG_WARP;
};

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
  // LM-head epilogues (C = hidden states x vocabulary rows):
  const int64_t* targets;  // [M] target vocabulary id of each row (<0: none)
  float4* stats;           // EPI_STATS: [M, num_n] (max, sum exp(x-max), sum exp(x-max) x, 0)
  float* tgt;              // EPI_STATS: [M] logit of the target (written by the tile holding it)
  const float* lse;        // EPI_GRAD: [M] log-sum-exp of the row
  const float* g;          // EPI_GRAD: [M] d loss / d logprob of the row
  // reduce-scatter epilogue (scatter_rows > 0): output rows [r*scatter_rows,
  // (r+1)*scatter_rows) go to rank r's staging buffer peer[r] (a peer-mapped
  // address) at row offset slot*scatter_rows, with row stride ldc
  int scatter_rows;
  int scatter_slot;
  long long peer[8];
};

// Epilogue variants of the pair GEMM.
//  EPI_STORE  C = acc (+ bias) (+ C), bf16
//  EPI_STATS  per row and 256-column tile, the online softmax partials of
//             the fp32 logits and the target logit; with C null nothing else
//             is stored (LM-head forward: the [M, N] logits never reach
//             memory), else the bf16 logits are stored as well (kept for a
//             backward that does not recompute them)
//  EPI_GRAD   C = g * (onehot(target) - exp(acc - lse)), bf16 (LM-head
//             backward: the logits tile is recomputed in TMEM and only its
//             gradient is written, for the input-gradient GEMM that follows)
//  EPI_NONE   the accumulator is released unread (a measurement of the
//             mainloop alone: operand delivery and MMA issue)
enum { EPI_STORE = 0, EPI_STATS = 1, EPI_GRAD = 2, EPI_NONE = 3 };

template <int TN>
__device__ __forceinline__ int2 pair_tile(int t, int num_m, int num_n, int group_m) {
  const int group = group_m * num_n;
  const int g = t / group;
  const int first_m = g * group_m;
  const int gm = min(num_m - first_m, group_m);
  const int r = t - g * group;
  return make_int2((first_m + r % gm) * PBM, (r / gm) * TN);
}

template <int EPI, int TN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(P_THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2,
                     const PairArgs p) {
  using T = PTile<TN>;
  constexpr int PSTAGES = T::STAGES, P_STAGE = T::STAGE, NB = T::NB, NBUF = T::NBUF;
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
  const int num_n = (p.N + TN - 1) / TN;
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
        const int2 c = pair_tile<TN>(t, num_m, num_n, p.group_m);
        const int am = c.x + (int)rank * 128;
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % PSTAGES;
          const uint32_t ph = (it / PSTAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.err, 21)) {
            ok = false;
            break;
          }
          uint8_t* a = smem + s * P_STAGE;
          const uint32_t fb = full_leader + s * 8;
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * P_STAGE);  // both CTAs' bytes
          if (kb < p.nk1) tma_load_2d_pair(a, &tmA, fb, kb * PBK, am);
          else tma_load_2d_pair(a, &tmA2, fb, (kb - p.nk1) * PBK, am);
#pragma unroll
          for (int h = 0; h < NB; ++h) {  // this CTA's 128 columns of each N=256 half
            uint8_t* b = a + P_HALF * (1 + h);
            const int bn = c.y + h * 256 + (int)rank * 128;
            if (kb < p.nk1) {
              if (p.b_mn) {  // two 64-column boxes of the [K, N] matrix: 64 K rows each
                tma_load_2d_pair(b, &tmB, fb, bn, kb * PBK);
                tma_load_2d_pair(b + P_HALF / 2, &tmB, fb, bn + 64, kb * PBK);
              } else {
                tma_load_2d_pair(b, &tmB, fb, kb * PBK, bn);
              }
            } else {
              tma_load_2d_pair(b, &tmB2, fb, (kb - p.nk1) * PBK, bn);
            }
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
        const int buf = NBUF == 2 ? (tl & 1) : 0;
        const uint32_t use = (uint32_t)(NBUF == 2 ? (tl >> 1) : tl);
        const uint64_t ta = p.diag ? gtimer() : 0;
        if (!mbar_wait(&acc_empty[buf], (use & 1) ^ 1, abort_flag, p.err, 22)) break;
        if (p.diag) d_acc += gtimer() - ta;
        tc_fence_after();
        const uint32_t d = tmem + buf * TN;  // half h accumulates at d + 256 h
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
          const uint64_t da = desc_k_sw128(a_addr);
          if (kb < p.nk1 && p.b_mn) {
            // MN-major B: 16 K rows of 128 B per step (+2048 B), 64-column chunks 8 KB apart
#pragma unroll
            for (int kk = 0; kk < PBK / 16; ++kk)
#pragma unroll
              for (int h = 0; h < NB; ++h)
                mma_bf16_pair(d + 256 * h, da + 2 * kk,
                              desc_mn_sw128(a_addr + P_HALF * (1 + h), P_HALF / 2) + 128 * kk,
                              idesc | (1u << 16), (kb > 0 || kk > 0) ? 1u : 0u);
          } else if (kb < p.nk1) {
#pragma unroll
            for (int kk = 0; kk < PBK / 16; ++kk)  // +32 bytes per K=16 step (descriptor units of 16 B)
#pragma unroll
              for (int h = 0; h < NB; ++h)
                mma_bf16_pair(d + 256 * h, da + 2 * kk, desc_k_sw128(a_addr + P_HALF * (1 + h)) + 2 * kk, idesc,
                              (kb > 0 || kk > 0) ? 1u : 0u);
          } else {
            const int rem = p.K2 - (kb - p.nk1) * PBK;
            const int ksteps = min(PBK / 16, (rem + 15) / 16);
            for (int kk = 0; kk < ksteps; ++kk)
#pragma unroll
              for (int h = 0; h < NB; ++h)
                mma_bf16_pair(d + 256 * h, da + 2 * kk, desc_k_sw128(a_addr + P_HALF * (1 + h)) + 2 * kk, idesc, 1u);
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
    uint8_t* stg = smem + PSTAGES * P_STAGE + 256 + (warp - 2) * P_STG_WARP;
    int tl = 0;
    for (int t = pair; t < num_tiles; t += npairs, ++tl) {
      const int buf = NBUF == 2 ? (tl & 1) : 0;
      const uint32_t use = (uint32_t)(NBUF == 2 ? (tl >> 1) : tl);
      if (!__all_sync(0xffffffffu, mbar_wait_sleep(&acc_full[buf], use & 1, abort_flag, p.err, 24))) break;
      tc_fence_after();
      if constexpr (EPI == EPI_NONE) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(acce_leader + buf * 8);
        continue;
      }
      const int2 c = pair_tile<TN>(t, num_m, num_n, p.group_m);
      const int row = c.x + (int)rank * 128 + q * 32 + lane;
      // LM-head epilogues: per-row inputs and the running softmax partials
      int64_t tgt_id = -1;
      float row_lse = 0.f, row_g = 0.f;
      float st_m = -INFINITY, st_s = 0.f, st_sx = 0.f;
      if constexpr (EPI != EPI_STORE) {
        if (row < p.M) {
          tgt_id = p.targets[row];
          if constexpr (EPI == EPI_GRAD) {
            row_lse = p.lse[row];
            row_g = p.g[row];
          }
        }
      }
#pragma unroll 1
      for (int cc = 0; cc < TN / 32; cc += 2) {
        uint32_t r2[2][32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + buf * TN + cc * 32, r2[0]);
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + buf * TN + (cc + 1) * 32, r2[1]);
        tmem_wait_ld();
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int col0 = c.y + (cc + h) * 32;
          if (row < p.M && col0 < p.N) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r2[h][j]);
            if constexpr (EPI == EPI_STATS) {
              // online softmax over this 32-column chunk (fp32 logits); the
              // max, the exponentials and the sums each run over independent
              // columns (four chains for the reductions) so latencies overlap
              float cm4[4] = {v[0], v[1], v[2], v[3]};
#pragma unroll
              for (int j = 4; j < 32; ++j) cm4[j & 3] = fmaxf(cm4[j & 3], v[j]);
              const float mn = fmaxf(st_m, fmaxf(fmaxf(cm4[0], cm4[1]), fmaxf(cm4[2], cm4[3])));
              const float sc = (st_m == -INFINITY) ? 0.f : __expf(st_m - mn);
              float e[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) e[j] = __expf(v[j] - mn);
              float s4[4] = {0.f, 0.f, 0.f, 0.f}, sx4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                s4[j & 3] += e[j];
                sx4[j & 3] = fmaf(e[j], v[j], sx4[j & 3]);
              }
              const int64_t rel = tgt_id - col0;
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (rel == j) p.tgt[row] = v[j];
              st_m = mn;
              st_s = fmaf(st_s, sc, (s4[0] + s4[1]) + (s4[2] + s4[3]));
              st_sx = fmaf(st_sx, sc, (sx4[0] + sx4[1]) + (sx4[2] + sx4[3]));
              if (p.C == nullptr) continue;  // statistics only; else the logits are stored too
            } else if constexpr (EPI == EPI_GRAD) {
              const int64_t rel = tgt_id - col0;
#pragma unroll
              for (int j = 0; j < 32; ++j)
                v[j] = row_g * ((rel == j ? 1.f : 0.f) - __expf(v[j] - row_lse));
            }
            if (EPI == EPI_STORE && p.bias) {
#pragma unroll
              for (int j = 0; j < 32; j += 8) {
                uint4 bv = *reinterpret_cast<const uint4*>(p.bias + col0 + j);
                const __nv_bfloat16* be = reinterpret_cast<const __nv_bfloat16*>(&bv);
#pragma unroll
                for (int e = 0; e < 8; ++e) v[j + e] += bf2f(be[e]);
              }
            }
            // bf16 into the warp's staging block: row = lane, 16-byte unit
            // u = 4h + j/8 of the 128-byte row, stored at unit u ^ (lane & 7)
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
              uint4 o;
              o.x = pack_bf16x2(v[j + 0], v[j + 1]);
              o.y = pack_bf16x2(v[j + 2], v[j + 3]);
              o.z = pack_bf16x2(v[j + 4], v[j + 5]);
              o.w = pack_bf16x2(v[j + 6], v[j + 7]);
              const int u = h * 4 + j / 8;
              *reinterpret_cast<uint4*>(stg + lane * 128 + ((u ^ (lane & 7)) << 4)) = o;
            }
          }
        }
        __syncwarp();
        // 4 rows x 128 contiguous bytes per store instruction
        const int cbase = c.y + cc * 32;
        const bool do_store = EPI != EPI_STATS || p.C != nullptr;
#pragma unroll
        for (int k = 0; k < 8 && do_store; ++k) {
          const int rr = 4 * k + (lane >> 3), u = lane & 7;
          const int grow = c.x + (int)rank * 128 + q * 32 + rr;
          const int gcol = cbase + u * 8;
          if (grow < p.M && gcol < p.N) {
            uint4 o = *reinterpret_cast<const uint4*>(stg + rr * 128 + ((u ^ (rr & 7)) << 4));
            __nv_bfloat16* dst;
            if (p.scatter_rows) {  // the owning rank's staging slot (P2P stores over NVLink)
              const int owner = grow / p.scatter_rows;
              dst = reinterpret_cast<__nv_bfloat16*>(p.peer[owner]) +
                    ((int64_t)p.scatter_slot * p.scatter_rows + (grow - owner * p.scatter_rows)) * p.ldc + gcol;
            } else {
              dst = p.C + (int64_t)grow * p.ldc + gcol;
            }
            if (EPI == EPI_STORE && p.accumulate_c) {  // out += product (a second bf16 rounding)
              const uint4 cv = *reinterpret_cast<const uint4*>(dst);
              const __nv_bfloat16* ce = reinterpret_cast<const __nv_bfloat16*>(&cv);
              const __nv_bfloat16* oe = reinterpret_cast<const __nv_bfloat16*>(&o);
              o.x = pack_bf16x2(bf2f(oe[0]) + bf2f(ce[0]), bf2f(oe[1]) + bf2f(ce[1]));
              o.y = pack_bf16x2(bf2f(oe[2]) + bf2f(ce[2]), bf2f(oe[3]) + bf2f(ce[3]));
              o.z = pack_bf16x2(bf2f(oe[4]) + bf2f(ce[4]), bf2f(oe[5]) + bf2f(ce[5]));
              o.w = pack_bf16x2(bf2f(oe[6]) + bf2f(ce[6]), bf2f(oe[7]) + bf2f(ce[7]));
            }
            *reinterpret_cast<uint4*>(dst) = o;
          }
        }
        __syncwarp();
      }
      if constexpr (EPI == EPI_STATS) {
        if (row < p.M) p.stats[(int64_t)row * num_n + c.y / TN] = make_float4(st_m, st_s, st_sx, 0.f);
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

// Merge of the per-tile softmax partials of the LM-head forward: one warp
// per row; lse = M + log S, entropy = lse - SX / S, logprob = x_target - lse.
__device__ __forceinline__ void part_merge(float& m, float& s, float& sx, float m2, float s2, float sx2) {
  if (m2 == -INFINITY) return;
  if (m == -INFINITY) {
    m = m2;
    s = s2;
    sx = sx2;
    return;
  }
  const float mn = fmaxf(m, m2);
  const float a = __expf(m - mn), b = __expf(m2 - mn);
  s = s * a + s2 * b;
  sx = sx * a + sx2 * b;
  m = mn;
}

__global__ void lm_head_merge_kernel(const float4* __restrict__ stats, int num_n, int M,
                                     const int64_t* __restrict__ targets, int V, const float* __restrict__ tgt,
                                     float* __restrict__ lp, float* __restrict__ ent, float* __restrict__ lse) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  float m = -INFINITY, s = 0.f, sx = 0.f;
  for (int i = lane; i < num_n; i += 32) {
    const float4 v = stats[(int64_t)row * num_n + i];
    part_merge(m, s, sx, v.x, v.y, v.z);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    const float sx2 = __shfl_xor_sync(0xffffffffu, sx, o);
    part_merge(m, s, sx, m2, s2, sx2);
  }
  if (lane == 0) {
    const float l = m + logf(s);
    lse[row] = l;
    if (ent) ent[row] = l - sx / s;
    const int64_t t = targets[row];
    lp[row] = ((t >= 0 && t < V) ? tgt[row] : 0.f) - l;
  }
}

template <int EPI, int TN>
int pair_capacity(int dev) {
  static int max_pairs[64] = {0};
  if (!max_pairs[dev]) {
    ART_CUDA_CHECK(cudaFuncSetAttribute(gemm_pair_kernel<EPI, TN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        PTile<TN>::SMEM));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(P_THREADS, 1, 1);
    cfg.dynamicSmemBytes = PTile<TN>::SMEM;  // cluster shape comes from __cluster_dims__
    int n = 0;
    ART_CUDA_CHECK(cudaOccupancyMaxActiveClusters(&n, gemm_pair_kernel<EPI, TN>, &cfg));
    TORCH_CHECK(n > 0, "no CTA pair of the GEMM fits on this device");
    max_pairs[dev] = n;
  }
  return max_pairs[dev];
}

// Tile width of a call: the 512-wide tile (less staging traffic per FLOP,
// one accumulator buffer) where its tile count fills the resident pairs about
// as evenly as the 256-wide one; ART_B200_PAIR_WIDE=0 / 1 forces 256 / 512.
constexpr int kPairWideDefault = -1;  // -1: chosen per call (ART_B200_PAIR_WIDE=0 / 1 force 256 / 512)

inline int pair_tile_n(int64_t M, int64_t N, int pairs) {
  const char* e = std::getenv("ART_B200_PAIR_WIDE");  // read per call: tests and benchmarks switch it
  const int force = e ? std::atoi(e) : kPairWideDefault;
  if (force == 0 || N < 512) return 256;
  if (force == 1) return 512;
  const double num_m = (double)((M + PBM - 1) / PBM);
  auto fill = [&](int64_t tn) {
    const double tiles = num_m * (double)((N + tn - 1) / tn);
    const double waves = tiles / pairs;
    return waves / std::ceil(waves);
  };
  // the wide tile's mainloop runs ~10 % faster when it is not limited by tile quantisation
  return fill(512) * 1.10 > fill(256) ? 512 : 256;
}

template <int EPI, int TN>
void launch_pair_tn(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ta2, const CUtensorMap& tb2,
                    PairArgs& p, int64_t K, int dev) {
  {
    const int64_t num_m = (p.M + PBM - 1) / PBM;
    const int64_t band = (int64_t)PBM * K * 2;  // bytes of one 256-row band of A
    int64_t g = ((int64_t)48 << 20) / (band > 0 ? band : 1);
    p.group_m = (int)std::max<int64_t>(1, std::min<int64_t>(g, num_m));
  }
  p.err = tc_error_ptr(dev);
  const int cap = pair_capacity<EPI, TN>(dev);
  const int tiles = ((p.M + PBM - 1) / PBM) * ((p.N + TN - 1) / TN);
  const int pairs = tiles < cap ? tiles : cap;
  gemm_pair_kernel<EPI, TN><<<2 * pairs, P_THREADS, PTile<TN>::SMEM, at::cuda::getCurrentCUDAStream()>>>(
      ta, tb, ta2, tb2, p);
  ART_CUDA_CHECK(cudaPeekAtLastError());
}

// Launch with the tile width chosen for the call (returned: the LM-head
// statistics are laid out per tile of that width).
template <int EPI>
int launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ta2, const CUtensorMap& tb2,
                PairArgs& p, int64_t K, int dev, int tn = 0) {
  if (!tn) tn = pair_tile_n(p.M, p.N, pair_capacity<EPI, 256>(dev));
  if (tn == 512) launch_pair_tn<EPI, 512>(ta, tb, ta2, tb2, p, K, dev);
  else launch_pair_tn<EPI, 256>(ta, tb, ta2, tb2, p, K, dev);
  return tn;
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
  p.targets = nullptr;
  p.stats = nullptr;
  p.tgt = nullptr;
  p.lse = nullptr;
  p.g = nullptr;
  p.scatter_rows = 0;
  p.scatter_slot = 0;
  for (int i = 0; i < 8; ++i) p.peer[i] = 0;
  launch_pair<EPI_STORE>(ta, tb, ta2, tb2, p, K, a.get_device());
  return c;
}

// RS(a @ b^T (+ a2 @ b2^T)): the product's row block r goes straight into
// rank r's staging slot `slot` (peer pointers c_ptrs, row stride ldc); the
// owner sums its slots afterwards.  Same contract as gemm_tc_rs, on CTA pairs.
void gemm_pair_rs(torch::Tensor a, torch::Tensor b, c10::optional<torch::Tensor> a2, c10::optional<torch::Tensor> b2,
                  std::vector<int64_t> c_ptrs, int64_t rows, int64_t ldc, int64_t slot) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && a.size(1) == b.size(1));
  const int64_t M = a.size(0), K = a.size(1), N = b.size(0);
  const int ndst = (int)c_ptrs.size();
  TORCH_CHECK(ndst >= 1 && ndst <= 8 && rows * ndst == M && N % 32 == 0 && ldc % 8 == 0);
  if (a2.has_value()) TORCH_CHECK(b2.has_value() && a2->size(0) == M && b2->size(0) == N && a2->size(1) == b2->size(1));
  const CUtensorMap ta = make_tmap_bf16(a, 128), tb = make_tmap_bf16(b, 128);
  const CUtensorMap ta2 = a2.has_value() ? make_tmap_bf16(*a2, 128) : ta;
  const CUtensorMap tb2 = a2.has_value() ? make_tmap_bf16(*b2, 128) : tb;
  PairArgs p;
  p.M = (int)M;
  p.N = (int)N;
  p.K2 = a2.has_value() ? (int)a2->size(1) : 0;
  p.nk1 = (int)((K + PBK - 1) / PBK);
  p.nk2 = a2.has_value() ? (p.K2 + PBK - 1) / PBK : 0;
  p.C = nullptr;
  p.ldc = ldc;
  p.bias = nullptr;
  p.accumulate_c = 0;
  p.b_mn = 0;
  p.diag = nullptr;
  p.targets = nullptr;
  p.stats = nullptr;
  p.tgt = nullptr;
  p.lse = nullptr;
  p.g = nullptr;
  p.scatter_rows = (int)rows;
  p.scatter_slot = (int)slot;
  for (int i = 0; i < 8; ++i) p.peer[i] = i < ndst ? c_ptrs[i] : 0;
  if (M == 0) return;
  launch_pair<EPI_STORE>(ta, tb, ta2, tb2, p, K, a.get_device());
}

// The mainloop alone (EPI_NONE) with the MMA-thread counters of PairArgs::diag:
// a measurement entry point for the benchmark suite.
void gemm_pair_mainloop(torch::Tensor a, torch::Tensor b, torch::Tensor diag) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && a.size(1) == b.size(1));
  TORCH_CHECK(diag.is_cuda() && diag.scalar_type() == torch::kInt64 && diag.numel() >= 5, "diag: int64[5]");
  const CUtensorMap ta = make_tmap_bf16(a, 128), tb = make_tmap_bf16(b, 128);
  PairArgs p;
  p.M = (int)a.size(0);
  p.N = (int)b.size(0);
  p.K2 = 0;
  p.nk1 = (int)((a.size(1) + PBK - 1) / PBK);
  p.nk2 = 0;
  p.C = nullptr;
  p.ldc = 0;
  p.bias = nullptr;
  p.accumulate_c = 0;
  p.b_mn = 0;
  p.diag = reinterpret_cast<unsigned long long*>(diag.data_ptr<int64_t>());
  p.targets = nullptr;
  p.stats = nullptr;
  p.tgt = nullptr;
  p.lse = nullptr;
  p.g = nullptr;
  p.scatter_rows = 0;
  p.scatter_slot = 0;
  for (int i = 0; i < 8; ++i) p.peer[i] = 0;
  launch_pair<EPI_NONE>(ta, tb, ta, tb, p, a.size(1), a.get_device());
}

static void lm_head_check(const torch::Tensor& h, const torch::Tensor& w, const torch::Tensor& targets) {
  TORCH_CHECK(h.is_cuda() && w.is_cuda() && targets.is_cuda(), "LM head: CUDA tensors");
  TORCH_CHECK(h.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "LM head: bf16 operands");
  TORCH_CHECK(h.dim() == 2 && w.dim() == 2 && h.size(1) == w.size(1), "LM head: h [M, H], w [V, H]");
  TORCH_CHECK(h.size(0) >= 128 && w.size(0) >= 128, "LM head: at least 128 rows and 128 vocabulary entries");
  TORCH_CHECK(w.size(0) % 32 == 0, "LM head: vocabulary size must be a multiple of 32");
  TORCH_CHECK(targets.scalar_type() == at::kLong && targets.is_contiguous() && targets.numel() == h.size(0));
}

static PairArgs lm_head_args(const torch::Tensor& h, const torch::Tensor& w) {
  PairArgs p;
  p.M = (int)h.size(0);
  p.N = (int)w.size(0);
  p.K2 = 0;
  p.nk1 = (int)((h.size(1) + PBK - 1) / PBK);
  p.nk2 = 0;
  p.C = nullptr;
  p.ldc = 0;
  p.bias = nullptr;
  p.accumulate_c = 0;
  p.b_mn = 0;
  p.diag = nullptr;
  p.targets = nullptr;
  p.stats = nullptr;
  p.tgt = nullptr;
  p.lse = nullptr;
  p.g = nullptr;
  p.scatter_rows = 0;
  p.scatter_slot = 0;
  for (int i = 0; i < 8; ++i) p.peer[i] = 0;
  return p;
}

// LM-head forward: per row, log softmax(h w^T)[target] (fp32 logits in TMEM),
// the entropy (if asked) and the log-sum-exp kept for the backward.  With
// logits_out ([M, V] bf16) the epilogue also stores the logits.
// Returns {logprob, entropy or undefined, lse}.
std::vector<torch::Tensor> lm_head_fwd(torch::Tensor h, torch::Tensor w, torch::Tensor targets, bool entropy,
                                       c10::optional<torch::Tensor> logits_out) {
  lm_head_check(h, w, targets);
  const int64_t M = h.size(0), V = w.size(0);
  const int tn = pair_tile_n(M, V, pair_capacity<EPI_STATS, 256>(h.get_device()));
  const int64_t num_n = (V + tn - 1) / tn;
  auto f32 = h.options().dtype(at::kFloat);
  auto stats = torch::empty({M, num_n, 4}, f32);
  auto tgt = torch::zeros({M}, f32);
  auto lp = torch::empty({M}, f32), lse = torch::empty({M}, f32);
  auto ent = entropy ? torch::empty({M}, f32) : torch::Tensor();
  const CUtensorMap ta = make_tmap_bf16(h, 128), tb = make_tmap_bf16(w, 128);
  PairArgs p = lm_head_args(h, w);
  p.targets = targets.data_ptr<int64_t>();
  p.stats = reinterpret_cast<float4*>(stats.data_ptr<float>());
  p.tgt = tgt.data_ptr<float>();
  if (logits_out.has_value()) {
    const auto& out = *logits_out;
    TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.size(0) == M && out.size(1) == V && out.stride(1) == 1 &&
                out.stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(out.data_ptr()) % 16) == 0,
                "logits_out: bf16 [M, V], 16-byte aligned rows");
    p.C = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
    p.ldc = out.stride(0);
  }
  launch_pair<EPI_STATS>(ta, tb, ta, tb, p, h.size(1), h.get_device(), tn);
  lm_head_merge_kernel<<<(unsigned)((M + 7) / 8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const float4*>(stats.data_ptr<float>()), (int)num_n, (int)M, targets.data_ptr<int64_t>(),
      (int)V, tgt.data_ptr<float>(), lp.data_ptr<float>(), entropy ? ent.data_ptr<float>() : nullptr,
      lse.data_ptr<float>());
  ART_CUDA_CHECK(cudaPeekAtLastError());
  return {lp, ent, lse};
}

// LM-head backward, first half: the logits of h w^T recomputed tile by tile
// in TMEM and turned into dlogits = g * (onehot(target) - softmax) in the
// epilogue; written into out [M, V] bf16 (the input gradient dh = dlogits w
// follows as a pair GEMM on w in its stored layout).
void lm_head_grad_logits(torch::Tensor h, torch::Tensor w, torch::Tensor targets, torch::Tensor lse, torch::Tensor g,
                         torch::Tensor out) {
  lm_head_check(h, w, targets);
  TORCH_CHECK(lse.scalar_type() == at::kFloat && g.scalar_type() == at::kFloat && lse.is_contiguous() &&
              g.is_contiguous() && lse.numel() == h.size(0) && g.numel() == h.size(0));
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.size(0) == h.size(0) && out.size(1) == w.size(0) &&
              out.stride(1) == 1 && out.stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(out.data_ptr()) % 16) == 0);
  const CUtensorMap ta = make_tmap_bf16(h, 128), tb = make_tmap_bf16(w, 128);
  PairArgs p = lm_head_args(h, w);
  p.C = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.ldc = out.stride(0);
  p.targets = targets.data_ptr<int64_t>();
  p.lse = lse.data_ptr<float>();
  p.g = g.data_ptr<float>();
  launch_pair<EPI_GRAD>(ta, tb, ta, tb, p, h.size(1), h.get_device());
}

}  // namespace art
