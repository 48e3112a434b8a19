// Expert-parallel MoE on sm_100a: the token dispatch fused with the grouped
// expert GEMM, and the combine fused into the grouped GEMM's epilogue.
//
// Reference behaviour: Megatron MoE with the DeepEP dispatcher around the
// experts' grouped GEMMs (src/art/megatron/provider.py:416-434,
// lora.py:1464-1572).  Here one persistent kernel per exchange does both the
// transfer and the math over NVLink peer memory:
//
//  ep_dispatch_gemm   every CTA runs the grouped tcgen05 GEMM of this rank's
//                     experts (warp 0 TMA, warp 1 MMA, warps 2-5 epilogue, as
//                     in gemm_tc.cu) while its warps 6-7 push this rank's
//                     token rows (and their rank-side LoRA rows) into the
//                     owners' receive buffers with 16-byte P2P stores.  Rows
//                     are pushed in (local expert, owner) order by the whole
//                     grid, so every owner's first experts complete first; a
//                     tile's TMA loads start as soon as its expert's arrival
//                     counter (bumped by the senders with release adds after
//                     each batch) reaches the expected row count: the GEMM
//                     overlaps the all-to-all tile by tile.
//  ep_gemm (scatter)  the grouped GEMM whose epilogue stores each output row
//                     straight into the origin rank's slot buffer (the row's
//                     (rank, slot) came with the dispatched row) and adds the
//                     rows it delivered to the origin's arrival counter.
//  ep_wait_combine    the origin waits for all its slots, then reduces the k
//                     slots of every token (weighted by the routing weights).
//
// Ordering rules that make the flags safe: every exchange starts after a
// peer barrier (so no rank writes into a buffer a slower rank still reads);
// counters only grow, and the host passes cumulative targets; every wait is
// bounded (%globaltimer) and records an error code instead of hanging.  No
// TMA load touches peer memory here: peers are written with plain stores and
// read locally.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <cudaTypedefs.h>
#include "common.cuh"
#include "tc_common.cuh"

namespace art {
using namespace tc;

namespace {
constexpr int XBM = 128, XBN = 256, XBK = 64, XSTAGES = 4;
constexpr int XA_TILE = XBM * XBK * 2;
constexpr int XB_TILE = XBN * XBK * 2;
constexpr int XSTAGE_BYTES = XA_TILE + XB_TILE;
constexpr int XTHREADS = 256;  // warps 0 TMA, 1 MMA, 2..5 epilogue, 6..7 dispatch
constexpr int X_STG_WARP = 32 * 128;  // epilogue staging per warp: 32 rows x 64 bf16
constexpr int XSMEM = XSTAGES * XSTAGE_BYTES + 1024 + 512 + 4 * X_STG_WARP;
constexpr int XMAX_RANKS = 8;
constexpr int PUSH_BATCH = 8;
constexpr int kPushSeg = 8;  // 16-byte loads in flight per lane while pushing a row
constexpr uint64_t kEpWaitNs = 3ull * 1000 * 1000 * 1000;
constexpr int kExtLd = 64;  // row stride (elements) of the receive buffer of rank-side rows

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Bounded wait until counter - target >= 0 (wrap-safe).
__device__ __forceinline__ bool wait_count(const uint32_t* ctr, uint32_t target, volatile int* abort_flag,
                                           int* err, int code) {
  const uint64_t t0 = gtimer();
  for (uint32_t it = 0;; ++it) {
    if ((int32_t)(ld_acquire_u32(ctr) - target) >= 0) return true;
    if ((it & 63) == 63) {
      if (abort_flag && *abort_flag) return false;
      if (gtimer() - t0 > kEpWaitNs) {
        if (abort_flag) *abort_flag = 1;
        if (err) atomicCAS(err, 0, code);
        return false;
      }
    }
    __nanosleep(40);
  }
}
}  // namespace

struct EpGemmArgs {
  int M, N, K2, nk1, nk2, b_mn, kmain;
  const int4* tiles;  // (m0, n0, row of B, end of the expert's rows)
  int num_tiles;
  int* err;
  // plain output
  __nv_bfloat16* C;
  int64_t ldc;
  // arrival waits: tile t reads the rows of local expert tile_expert[t]
  const int* tile_expert;
  const uint32_t* arrive_local;   // this rank's per-local-expert counters
  const uint32_t* arrive_target;  // cumulative targets
  // dispatch (push) phase, in push order
  int n_push, H, ext_cols, world;
  const __nv_bfloat16* src;  // token rows [*, H] (row stride ld_src)
  int64_t ld_src;
  const __nv_bfloat16* src_ext;  // [n_push, ext_cols] rank-side rows (push order) or null
  const int64_t* push_tok;
  const float* push_scale;
  const int* push_rank;
  const int64_t* push_row;
  const int* push_expert;
  const int64_t* push_meta;  // value stored in the owner's row meta (origin rank << 40 | slot)
  long long recv_x[XMAX_RANKS], recv_ext[XMAX_RANKS], recv_meta[XMAX_RANKS], arrive[XMAX_RANKS];
  // scattered epilogue: row -> (origin rank << 40 | slot row); null = plain C
  const int64_t* row_dst;
  long long slot_base[XMAX_RANKS];
  long long slot_count[XMAX_RANKS];
};

__global__ void __launch_bounds__(XTHREADS, 1)
    ep_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2,
                   const EpGemmArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + XSTAGES * XSTAGE_BYTES);
  uint64_t* empty = full + XSTAGES;
  uint64_t* acc_full = empty + XSTAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* cnt = reinterpret_cast<int*>(tmem_slot + 2);  // [2][XMAX_RANKS] rows delivered per origin
  int* done = cnt + 2 * XMAX_RANKS;                                           // [2] epilogue warps done

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = p.nk1 + p.nk2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < XSTAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    *abort_flag = 0;
    for (int i = 0; i < 2 * XMAX_RANKS + 2; ++i) cnt[i] = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0 && p.num_tiles > 0) {
      prefetch_tmap(&tmA);
      prefetch_tmap(&tmB);
      if (p.nk2) {
        prefetch_tmap(&tmA2);
        prefetch_tmap(&tmB2);
      }
      int it = 0, waited = -1;
      for (int tile = blockIdx.x; tile < p.num_tiles && !*abort_flag; tile += gridDim.x) {
        const int4 tc4 = __ldg(p.tiles + tile);
        const int m0 = tc4.x, n0 = tc4.y, brow = tc4.z;
        if (p.tile_expert) {
          const int e = __ldg(p.tile_expert + tile);
          if (e >= 0 && e != waited) {
            // the expert's rows (and their metadata) have all landed
            if (!wait_count(p.arrive_local + e, __ldg(p.arrive_target + e), abort_flag, p.err, 5)) break;
            fence_proxy_async_global();  // generic-proxy peer writes -> visible to TMA reads
            waited = e;
          }
        }
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % XSTAGES;
          const uint32_t ph = (it / XSTAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.err, 1)) break;
          uint8_t* a = smem + s * XSTAGE_BYTES;
          uint8_t* b = a + XA_TILE;
          mbar_arrive_expect_tx(&full[s], XSTAGE_BYTES);
          if (kb < p.nk1) {
            tma_load_2d(a, &tmA, &full[s], kb * XBK, m0);
            if (p.b_mn) {
#pragma unroll
              for (int j = 0; j < XBN / 64; ++j)
                tma_load_2d(b + j * (XBK * 128), &tmB, &full[s], n0 + 64 * j, brow + kb * XBK);
            } else {
              tma_load_2d(b, &tmB, &full[s], kb * XBK, brow);
            }
          } else {
            const int k2 = (kb - p.nk1) * XBK;
            const int b2row = p.b_mn ? (brow / p.kmain) * p.N + n0 : brow;
            tma_load_2d(a, &tmA2, &full[s], k2, m0);
            tma_load_2d(b, &tmB2, &full[s], k2, b2row);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(XBM, XBN);
      int it = 0, t = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles && !*abort_flag; tile += gridDim.x, ++t) {
        const int buf = t & 1;
        const uint32_t use = (uint32_t)(t >> 1);
        if (!mbar_wait(&acc_empty[buf], (use & 1) ^ 1, abort_flag, p.err, 2)) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * XBN;
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % XSTAGES;
          const uint32_t ph = (it / XSTAGES) & 1;
          if (!mbar_wait(&full[s], ph, abort_flag, p.err, 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_addr(smem + s * XSTAGE_BYTES);
          const uint32_t b_addr = a_addr + XA_TILE;
          int ksteps = XBK / 16;
          if (kb >= p.nk1) {
            const int rem = p.K2 - (kb - p.nk1) * XBK;
            ksteps = min(ksteps, (rem + 15) / 16);
          }
          const bool bmn = p.b_mn && kb < p.nk1;
          for (int kk = 0; kk < ksteps; ++kk)
            mma_bf16(d, desc_k_sw128(a_addr + kk * 32),
                     bmn ? desc_mn_sw128(b_addr + kk * 2048, XBK * 128) : desc_k_sw128(b_addr + kk * 32),
                     bmn ? (idesc | (1u << 16)) : idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&empty[s]);
        }
        if (!ok) break;
        mma_commit(&acc_full[buf]);
      }
    }
  } else if (warp <= 5) {
    // epilogue warps 2..5 -> TMEM lane quadrants 2,3,0,1
    const int q = warp & 3;
    int t = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++t) {
      const int buf = t & 1;
      const uint32_t use = (uint32_t)(t >> 1);
      if (!mbar_wait_warp(&acc_full[buf], use & 1, abort_flag, p.err, 4)) break;
      tc_fence_after();
      const int4 tc4 = __ldg(p.tiles + tile);
      const int m0 = tc4.x, n0 = tc4.y, row_end = tc4.w;
      const int row = m0 + q * 32 + lane;
      const bool valid = row < row_end;
      __nv_bfloat16* dst_row = nullptr;
      int origin = -1;
      if (valid) {
        if (p.row_dst) {
          const int64_t d = p.row_dst[row];
          origin = (int)(d >> 40);
          const int64_t slot = d & ((int64_t(1) << 40) - 1);
          dst_row = reinterpret_cast<__nv_bfloat16*>(p.slot_base[origin]) + slot * p.ldc;
        } else {
          dst_row = p.C + (int64_t)row * p.ldc;
        }
      }
      // 64 columns per pass through the warp's staging block (16-byte units
      // XOR-swizzled by row), then 4 rows x 128 contiguous bytes per store
      // instruction: whole lines into the (local or peer) destination rows
      uint8_t* stg = smem + XSTAGES * XSTAGE_BYTES + 512 + (warp - 2) * X_STG_WARP;
#pragma unroll 1
      for (int c = 0; c < XBN / 32; c += 2) {
        uint32_t r[2][32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + buf * XBN + c * 32, r[0]);
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + buf * XBN + (c + 1) * 32, r[1]);
        tmem_wait_ld();
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            uint4 o;
            o.x = pack_bf16x2(__uint_as_float(r[h][j + 0]), __uint_as_float(r[h][j + 1]));
            o.y = pack_bf16x2(__uint_as_float(r[h][j + 2]), __uint_as_float(r[h][j + 3]));
            o.z = pack_bf16x2(__uint_as_float(r[h][j + 4]), __uint_as_float(r[h][j + 5]));
            o.w = pack_bf16x2(__uint_as_float(r[h][j + 6]), __uint_as_float(r[h][j + 7]));
            const int u = h * 4 + j / 8;
            *reinterpret_cast<uint4*>(stg + lane * 128 + ((u ^ (lane & 7)) << 4)) = o;
          }
        __syncwarp();
        const int cbase = n0 + c * 32;
        const uint64_t my_dst = reinterpret_cast<uint64_t>(dst_row);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int rr = 4 * k + (lane >> 3), u = lane & 7;
          const uint64_t dr = __shfl_sync(0xffffffffu, my_dst, rr);
          const int gcol = cbase + u * 8;
          if (dr != 0 && gcol < p.N) {
            const uint4 o = *reinterpret_cast<const uint4*>(stg + rr * 128 + ((u ^ (rr & 7)) << 4));
            *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(dr) + gcol) = o;
          }
        }
        __syncwarp();
      }
      if (p.row_dst) {
        // publish the delivered rows: each thread's stores, then one release
        // add per origin rank by the last epilogue warp to finish the tile
        __threadfence_system();
        const int par = t & 1;
        if (origin >= 0) atomicAdd(&cnt[par * XMAX_RANKS + origin], 1);
        __threadfence_block();
        __syncwarp();
        if (lane == 0) {
          const int old = atomicAdd(&done[par], 1);
          if (old == 3) {
            __threadfence_block();
            for (int i = 0; i < p.world; ++i) {
              const int v = atomicExch(&cnt[par * XMAX_RANKS + i], 0);
              if (v) red_release_add(reinterpret_cast<uint32_t*>(p.slot_count[i]), (uint32_t)v);
            }
            atomicExch(&done[par], 0);
          }
        }
        __syncwarp();
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
    }
  } else {
    // warps 6..7: dispatch this rank's rows to the owners (push order)
    const int pw = (warp - 6) + 2 * blockIdx.x;
    const int npw = 2 * gridDim.x;
    const int nbatch = (p.n_push + PUSH_BATCH - 1) / PUSH_BATCH;
    for (int b = pw; b < nbatch; b += npw) {
      const int i0 = b * PUSH_BATCH, i1 = min(i0 + PUSH_BATCH, p.n_push);
      for (int i = i0; i < i1; ++i) {
        const int rk = __ldg(p.push_rank + i);
        const int64_t row = __ldg(p.push_row + i);
        const __nv_bfloat16* s = p.src + __ldg(p.push_tok + i) * p.ld_src;
        __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(p.recv_x[rk]) + row * p.H;
        const float sc = p.push_scale ? __ldg(p.push_scale + i) : 1.f;
        // a segment of up to 2048 elements per pass: all of a lane's loads
        // are issued before its stores, so a warp waits one memory latency
        // per segment instead of one per 512-byte chunk
        for (int c0 = 0; c0 < p.H; c0 += kPushSeg * 256) {
          uint4 v[kPushSeg];
#pragma unroll
          for (int u = 0; u < kPushSeg; ++u) {
            const int c = c0 + u * 256 + lane * 8;
            if (c < p.H) v[u] = __ldg(reinterpret_cast<const uint4*>(s + c));
          }
#pragma unroll
          for (int u = 0; u < kPushSeg; ++u) {
            const int c = c0 + u * 256 + lane * 8;
            if (c < p.H) {
              if (p.push_scale) {
                __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&v[u]);
#pragma unroll
                for (int k = 0; k < 8; ++k) e[k] = f2bf(bf2f(e[k]) * sc);
              }
              *reinterpret_cast<uint4*>(d + c) = v[u];
            }
          }
        }
        if (p.src_ext) {
          const __nv_bfloat16* se = p.src_ext + (int64_t)i * p.ext_cols;
          __nv_bfloat16* de = reinterpret_cast<__nv_bfloat16*>(p.recv_ext[rk]) + row * kExtLd;
          for (int c = lane * 8; c < p.ext_cols; c += 256)
            *reinterpret_cast<uint4*>(de + c) = *reinterpret_cast<const uint4*>(se + c);
        }
        if (p.push_meta && lane == 0)
          reinterpret_cast<int64_t*>(p.recv_meta[rk])[row] = __ldg(p.push_meta + i);
      }
      __threadfence_system();
      __syncwarp();
      if (lane == 0) {
        // one release add per run of equal (owner, expert) inside the batch
        int i = i0;
        while (i < i1) {
          const int rk = __ldg(p.push_rank + i), e = __ldg(p.push_expert + i);
          int j = i + 1;
          while (j < i1 && __ldg(p.push_rank + j) == rk && __ldg(p.push_expert + j) == e) ++j;
          red_release_add(reinterpret_cast<uint32_t*>(p.arrive[rk]) + e, (uint32_t)(j - i));
          i = j;
        }
      }
      __syncwarp();
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Origin side of the fused combine: wait for every slot, then
// out[t] = sum_j w[t, j] * slots[t*k + j] (fp32 accumulate).
__global__ void ep_wait_combine_kernel(const __nv_bfloat16* __restrict__ slots, const float* __restrict__ w,
                                       int64_t T, int k, int H, __nv_bfloat16* __restrict__ out,
                                       const uint32_t* __restrict__ counter, uint32_t target, int* err) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = wait_count(counter, target, nullptr, err, 6) ? 1 : 0;
  __syncthreads();
  if (!ok) return;
  const int lane = threadIdx.x & 31;
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T;
       t += (int64_t)gridDim.x * (blockDim.x >> 5)) {
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
}

// ---------------------------------------------------------------- host side
static void fill_tables(EpGemmArgs& p, const std::vector<int64_t>& offs, int64_t N, int64_t K, bool w_transposed,
                        std::vector<int32_t>& tab, std::vector<int32_t>& tex) {
  const int64_t E = (int64_t)offs.size() - 1;
  for (int64_t e = 0; e < E; ++e) {
    TORCH_CHECK(offs[e + 1] >= offs[e], "offsets must be non-decreasing");
    for (int64_t n0 = 0; n0 < N; n0 += XBN)
      for (int64_t m0 = offs[e]; m0 < offs[e + 1]; m0 += XBM) {
        tab.push_back((int32_t)m0);
        tab.push_back((int32_t)n0);
        tab.push_back((int32_t)(w_transposed ? e * K : e * N + n0));
        tab.push_back((int32_t)offs[e + 1]);
        tex.push_back((int32_t)e);
      }
  }
  (void)p;
}

static torch::Tensor pinned_i32(const std::vector<int32_t>& v, const torch::Device& dev) {
  auto h = torch::from_blob(const_cast<int32_t*>(v.data()), {(int64_t)v.size()}, torch::kInt32).pin_memory();
  return h.to(dev, true);
}

// One fused exchange + grouped GEMM.
//   x [cap, K]        this rank's receive buffer (rows [0, offs[E]) valid after the waits)
//   w                 stacked expert weights ([E*N, K], or [E*K, N] with w_transposed)
//   offs              host offsets of the local experts' rows in x
//   a2 / b2           K-extension (LoRA) operands: a2 [cap, K2] (receive buffer of the
//                     rank-side rows), b2 [E*N, K2]
//   push_*            this rank's rows to send (push order), n = push_tok.numel()
//   recv_*_ptrs       per-rank base addresses of the receive buffers / counters
//   arrive_local / arrive_target  this rank's counters and cumulative targets
//   out               local output [cap, N] (plain mode) or, with row_dst, the rows go
//                     to slot_ptrs[origin] + slot * N and slot_count_ptrs[origin] is bumped.
void ep_gemm(torch::Tensor x, torch::Tensor w, std::vector<int64_t> offs, int64_t N, bool w_transposed,
             c10::optional<torch::Tensor> a2, c10::optional<torch::Tensor> b2,
             // dispatch
             c10::optional<torch::Tensor> src, c10::optional<torch::Tensor> src_ext,
             c10::optional<torch::Tensor> push_tok, c10::optional<torch::Tensor> push_scale,
             c10::optional<torch::Tensor> push_rank, c10::optional<torch::Tensor> push_row,
             c10::optional<torch::Tensor> push_expert, c10::optional<torch::Tensor> push_meta,
             std::vector<int64_t> recv_x_ptrs, std::vector<int64_t> recv_ext_ptrs, std::vector<int64_t> recv_meta_ptrs,
             std::vector<int64_t> arrive_ptrs, c10::optional<torch::Tensor> arrive_local,
             c10::optional<torch::Tensor> arrive_target,
             // output
             c10::optional<torch::Tensor> out, c10::optional<torch::Tensor> row_dst,
             std::vector<int64_t> slot_ptrs, std::vector<int64_t> slot_count_ptrs) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && x.dim() == 2 && w.dim() == 2);
  const int64_t K = x.size(1);
  const int64_t E = (int64_t)offs.size() - 1;
  TORCH_CHECK(E >= 1 && offs[0] == 0 && offs[E] <= x.size(0), "offsets must lie inside the receive buffer");
  if (w_transposed) {
    TORCH_CHECK(w.size(0) == E * K && w.size(1) == N && N % 64 == 0, "w must be [E*K, N]");
  } else {
    TORCH_CHECK(w.size(0) == E * N && w.size(1) == K && N % 32 == 0, "w must be [E*N, K]");
  }
  EpGemmArgs p;
  memset(&p, 0, sizeof(p));
  p.M = (int)offs[E];
  p.N = (int)N;
  p.K2 = a2.has_value() ? (int)a2->size(1) : 0;
  p.nk1 = (int)((K + XBK - 1) / XBK);
  p.nk2 = a2.has_value() ? (p.K2 + XBK - 1) / XBK : 0;
  p.b_mn = w_transposed ? 1 : 0;
  p.kmain = (int)K;
  if (a2.has_value()) TORCH_CHECK(b2.has_value() && b2->size(0) == E * N && a2->size(1) == b2->size(1));
  const int world = (int)std::max(recv_x_ptrs.size(), slot_ptrs.size());
  TORCH_CHECK(world <= XMAX_RANKS);
  p.world = world;
  // tile table (host offsets: the routing plan is known on the host)
  std::vector<int32_t> tab, tex;
  fill_tables(p, offs, N, K, w_transposed, tab, tex);
  const auto dev = x.device();
  torch::Tensor d_tab, d_tex;
  p.num_tiles = (int)tex.size();
  if (p.num_tiles) {
    d_tab = pinned_i32(tab, dev);
    p.tiles = reinterpret_cast<const int4*>(d_tab.data_ptr<int>());
  }
  // waits
  if (arrive_local.has_value()) {
    TORCH_CHECK(arrive_target.has_value() && arrive_local->numel() >= E && arrive_target->numel() >= E);
    d_tex = pinned_i32(tex, dev);
    p.tile_expert = p.num_tiles ? d_tex.data_ptr<int>() : nullptr;
    p.arrive_local = reinterpret_cast<const uint32_t*>(arrive_local->data_ptr<int>());
    p.arrive_target = reinterpret_cast<const uint32_t*>(arrive_target->data_ptr<int>());
  }
  // dispatch
  if (push_tok.has_value()) {
    TORCH_CHECK(src.has_value() && push_rank.has_value() && push_row.has_value() && push_expert.has_value());
    TORCH_CHECK(src->scalar_type() == at::kBFloat16 && src->stride(1) == 1 && src->size(1) == K && K % 8 == 0);
    p.n_push = (int)push_tok->numel();
    p.H = (int)K;
    p.src = reinterpret_cast<const __nv_bfloat16*>(src->data_ptr());
    p.ld_src = src->stride(0);
    p.push_tok = push_tok->data_ptr<int64_t>();
    p.push_rank = push_rank->data_ptr<int>();
    p.push_row = push_row->data_ptr<int64_t>();
    p.push_expert = push_expert->data_ptr<int>();
    p.push_scale = push_scale.has_value() ? push_scale->data_ptr<float>() : nullptr;
    p.push_meta = push_meta.has_value() ? push_meta->data_ptr<int64_t>() : nullptr;
    if (src_ext.has_value()) {
      TORCH_CHECK(src_ext->is_contiguous() && src_ext->size(0) >= p.n_push && src_ext->size(1) % 8 == 0 &&
                  src_ext->size(1) <= kExtLd);
      TORCH_CHECK((int)recv_ext_ptrs.size() == world);
      p.src_ext = reinterpret_cast<const __nv_bfloat16*>(src_ext->data_ptr());
      p.ext_cols = (int)src_ext->size(1);
    }
    TORCH_CHECK((int)arrive_ptrs.size() == world && (!p.push_meta || (int)recv_meta_ptrs.size() == world));
    for (int r = 0; r < world; ++r) {
      p.recv_x[r] = recv_x_ptrs[r];
      p.arrive[r] = arrive_ptrs[r];
      if (p.src_ext) p.recv_ext[r] = recv_ext_ptrs[r];
      if (p.push_meta) p.recv_meta[r] = recv_meta_ptrs[r];
    }
  }
  // output
  if (row_dst.has_value()) {
    TORCH_CHECK(row_dst->scalar_type() == at::kLong && row_dst->numel() >= p.M);
    TORCH_CHECK((int)slot_ptrs.size() == world && (int)slot_count_ptrs.size() == world);
    p.row_dst = row_dst->data_ptr<int64_t>();
    p.ldc = N;
    for (int r = 0; r < world; ++r) {
      p.slot_base[r] = slot_ptrs[r];
      p.slot_count[r] = slot_count_ptrs[r];
    }
  } else {
    TORCH_CHECK(out.has_value() && out->size(0) >= p.M && out->size(1) == N && out->stride(1) == 1 &&
                out->stride(0) % 8 == 0);
    p.C = reinterpret_cast<__nv_bfloat16*>(out->data_ptr());
    p.ldc = out->stride(0);
  }
  if (p.num_tiles == 0 && p.n_push == 0) return;
  // tensor maps (local memory only)
  auto xv = x.narrow(0, 0, std::max<int64_t>(p.M, 1));
  CUtensorMap ta = make_tmap_bf16(xv, XBM);
  CUtensorMap tb = make_tmap_bf16(w, w_transposed ? XBK : XBN);
  CUtensorMap ta2 = a2.has_value() ? make_tmap_bf16(a2->narrow(0, 0, std::max<int64_t>(p.M, 1)), XBM) : ta;
  CUtensorMap tb2 = a2.has_value() ? make_tmap_bf16(*b2, XBN) : tb;
  int dv = x.get_device();
  p.err = tc_error_ptr(dv);
  static int num_sms = 0;
  if (!num_sms) ART_CUDA_CHECK(cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dv));
  static bool attr = false;
  if (!attr) {
    ART_CUDA_CHECK(cudaFuncSetAttribute(ep_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, XSMEM));
    attr = true;
  }
  // persistent grid: one CTA per SM (every CTA also pushes its share of the rows)
  int grid = num_sms;
  if (p.n_push == 0) grid = std::min(grid, std::max(p.num_tiles, 1));
  ep_gemm_kernel<<<grid, XTHREADS, XSMEM, at::cuda::getCurrentCUDAStream()>>>(ta, tb, ta2, tb2, p);
  ART_CUDA_CHECK(cudaGetLastError());
}

torch::Tensor ep_wait_combine(torch::Tensor slots, c10::optional<torch::Tensor> w, int64_t k, torch::Tensor counter,
                              int64_t target) {
  TORCH_CHECK(slots.is_contiguous() && slots.scalar_type() == at::kBFloat16 && slots.size(1) % 8 == 0);
  const int H = slots.size(1);
  const int64_t T = slots.size(0) / k;
  auto out = torch::empty({T, H}, slots.options());
  if (w.has_value()) TORCH_CHECK(w->scalar_type() == at::kFloat && w->is_contiguous() && w->numel() >= T * k);
  int blocks = (int)std::min<int64_t>((T + 7) / 8, 148 * 4);
  if (blocks < 1) blocks = 1;
  ep_wait_combine_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(slots.data_ptr()), w.has_value() ? w->data_ptr<float>() : nullptr, T,
      (int)k, H, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
      reinterpret_cast<const uint32_t*>(counter.data_ptr<int>()), (uint32_t)(target & 0xffffffff),
      tc_error_ptr(slots.get_device()));
  ART_CUDA_CHECK(cudaGetLastError());
  return out;
}

}  // namespace art
