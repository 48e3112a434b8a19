// Prefix-tree attention forward on the 5th-generation tensor cores (sm_100a):
// tcgen05.mma with TMEM accumulators, TMA-fed shared memory, one elected
// thread issuing the MMAs.  Same contract as the warp-level kernel in
// attention.cu (GQA, head_dim 128, bf16 in, natural-log LSE out, mask
// "key j visible to query i iff j <= i < kend[j]", queries at global
// positions q_off + row).
//
// CTA = 128 queries x one q head; key tiles of 128, only the tiles whose
// largest kend reaches the query block are visited.
//   warp 0      TMA producer: Q once (2 boxes of 64 columns), then K and V of
//               every visited key tile into separate 2-stage rings (128-byte
//               swizzle): a K slot is released when S of its tile completes,
//               a V slot when P V completes, so the loads run ahead of the
//               tensor cores instead of sitting on the per-tile critical path
//   warp 1      TMEM allocation (512 columns) and the MMA issuer:
//                 S[b] = Q K^T         (M=128, N=128, K=128; both K-major,
//                                       b = tile mod 3)
//                 O   += P V           (P read from TMEM, where the softmax
//                                       stored it over S[b]; V MN-major
//                                       straight from its TMA tile)
//               issued as S(0), S(1), then S(n+2), P V(n) per tile: with
//               three S buffers the scores of the next two tiles are computed
//               while the softmax runs, and S(n+2) overwrites the buffer of
//               tile n-1 right after issuing its P V (tcgen05.mma operations
//               of one thread execute in order); the commit after P V
//               releases the V slot
//   warps 2..9  softmax, two warps per TMEM lane quadrant (one query row per
//               thread, each warp 64 of the 128 key columns and 64 of the
//               output columns): read the S half-row (tcgen05.ld), mask
//               (kend of partially visible tiles staged per warp in shared
//               memory, loaded while the warp waits for S),
//               running max (exchanged with the partner warp through a
//               bounded mbarrier handshake) with lazy rescaling of O (only
//               when the max grows by more than 2^8, the only time the
//               softmax waits for the previous P V), exp2, row sum, P as
//               bf16 pairs into the first 32 columns of the warp's S columns
//               (tcgen05.st); finally O / l to global memory and the LSE.
// TMEM columns: S[0] 0..127, S[1] 128..255, S[2] 256..383, O 384..511.
// All mbarrier waits are bounded (tc_common.cuh): on timeout the kernel
// records an error code, every role leaves its loop and TMEM is freed.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <cudaTypedefs.h>
#include "common.cuh"
#include "tc_common.cuh"

namespace art {
using namespace tc;

namespace {

constexpr int FB = 128;                      // queries per CTA = keys per tile = head_dim
constexpr int CHUNK_BYTES = FB * 64 * 2;     // 128 rows x 64 bf16 (one 128-byte swizzle span)
constexpr int TILE_BYTES = 2 * CHUNK_BYTES;  // 128 x 128 bf16
constexpr int KV_STAGES = 2;
constexpr int OFF_Q = 0;
constexpr int OFF_K = TILE_BYTES;                       // K stage s at OFF_K + s*T
constexpr int OFF_V = OFF_K + KV_STAGES * TILE_BYTES;  // V stage s at OFF_V + s*T
constexpr int OFF_P = OFF_V + KV_STAGES * TILE_BYTES;
constexpr int OFF_BAR = OFF_P + TILE_BYTES;
constexpr int MAX_KT = 1024;                 // key tiles per row the tile list holds (131072 keys)
constexpr int OFF_TL = OFF_BAR + 256;        // visible key-tile list (+ count)
constexpr int OFF_X = OFF_TL + MAX_KT * 4 + 16;  // exchange [3][2 half][128]: row max (2 parities), row sum
constexpr int OFF_KE = OFF_X + 3 * 2 * FB * 4;    // per softmax warp: kend of its 64 keys of the current tile
constexpr int FA_SMEM = OFF_KE + 8 * 64 * 4 + 1024;  // + alignment slack
constexpr int FA_NS = 3;                          // S / P buffers in tensor memory (O after them)
constexpr int TILE_FULL = 1 << 30;           // list flag: every (query, key) pair of the tile is visible
// 2 control warps + 8 softmax warps: two warps per TMEM lane quadrant, each
// owning 64 of a row's 128 key columns (and 64 of its 128 output columns)
constexpr int FA_THREADS = 320;
constexpr int FA_SOFT = 256;
constexpr float kLog2eF = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
constexpr int kExp2PolyEvery = 8;           // softmax: one exponent pair in 8 on the FMA pipe

// 2^x on the FMA pipe (x <= 2^22): x = r + f with r = round(x) (the 1.5 * 2^23
// shifter leaves r in the low mantissa bits), 2^f for f in [-1/2, 1/2] from a
// cubic with constant term 1 whose other coefficients were fitted for minimum
// maximum relative error on that interval (Lawson's iteratively reweighted
// least squares, 20001 points; relative error <= 1.02e-4, far below the
// bf16 rounding of P), and 2^r added to the exponent field.  Arguments below
// -127 are clamped there, which reconstructs exactly +0.
__device__ __forceinline__ float exp2_poly(float x) {
  x = fmaxf(x, -127.f);
  const float t = x + 12582912.f;
  const float f = x - (t - 12582912.f);
  const float q = fmaf(fmaf(fmaf(0.05500869f, f, 0.24221063f), f, 0.69328290f), f, 1.f);
  return __int_as_float(__float_as_int(q) + (__float_as_int(t) << 23));
}

struct FaArgs {
  const int* kend;
  const int* tile_kmax;  // max kend over 64-key tiles
  const int* tile_kmin;  // min kend over 64-key tiles
  __nv_bfloat16* o;
  int64_t ldo;
  float* lse;
  int Tq, Tk, q_off, Hq, Hkv;
  float scale_log2;
  int* err;
  // sliding window (window > 0): key j is visible to query i only if also
  // pos[i] - pos[j] < window (token positions, [Tk]); tile_pmax = max position
  // over each 128-key tile (tiles wholly out of the window are skipped)
  const int* pos;
  const int* tile_pmax;
  int window;
  // attention sinks (null: none): one logit per q head (natural-log units)
  // that joins every row's softmax denominator and attends to nothing
  const float* sinks;
  // phase clocks per CTA (null: off), kFaDiag int64 slots each: see attn_fwd_tc
  long long* diag;
};
constexpr int kFaDiag = 96;

// Visibility of key tile kt (128 keys) for the query block starting at global
// position g0: some key of the tile has kend > g0.
__device__ __forceinline__ bool tile_visible(const FaArgs& p, int kt, int g0) {
  const int a = 2 * kt, b = 2 * kt + 1;
  int km = __ldg(p.tile_kmax + a);
  if (b * 64 < p.Tk) km = max(km, __ldg(p.tile_kmax + b));
  return km > g0;
}

// Every pair of the (query block [g0, g_last], key tile kt) is visible: all
// keys precede the first query and every key's kend exceeds the last query.
__device__ __forceinline__ bool tile_full(const FaArgs& p, int kt, int g0, int g_last) {
  const int k_last = kt * FB + FB - 1;
  if (k_last >= p.Tk || k_last > g0) return false;
  const int km = min(__ldg(p.tile_kmin + 2 * kt), __ldg(p.tile_kmin + 2 * kt + 1));
  return km > g_last;
}

}  // namespace

// DIAG: the phase-clock build (FaArgs::diag), kept out of the production
// instance so that its code does not take instruction-cache space there
template <bool DIAG>
__global__ void __launch_bounds__(FA_THREADS, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const FaArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* k_empty = bars + 3;   // [2]
  uint64_t* v_full = bars + 5;    // [2]
  uint64_t* v_empty = bars + 7;   // [2]
  uint64_t* s_full = bars + 9;    // [FA_NS]: S of tile m completes phase (m/3)&1 of s_full[m%3]
  // [FA_NS]: P of tile m (all softmax threads) completes phase (m/3)&1 of
  // p_full[m%3]; one barrier per S buffer, as the softmax may finish tile
  // m+1 before the MMA thread has waited for tile m
  uint64_t* p_full = bars + 15;
  uint64_t* pv_done = bars + 18;  // [FA_NS]: P V of tile m completes phase (m/3)&1 of pv_done[m%3]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 21);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* xbar = bars + 23;  // [4]: the two softmax warps of a lane quadrant exchange row max / sum

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * FB;  // local query row of the block
  const int h = blockIdx.y;
  const int hk = h / (p.Hq / p.Hkv);
  const int g0 = p.q_off + q0;  // global position of the first query
  const int g_last = min(g0 + FB - 1, p.q_off + p.Tq - 1);
  const int kt_last = min(g_last / FB, (p.Tk - 1) / FB);
  long long* dg = DIAG ? p.diag + (int64_t)(blockIdx.y * gridDim.x + blockIdx.x) * kFaDiag : nullptr;
  auto tick = [&]() -> long long { return DIAG ? (long long)clock64() : 0ll; };

  if (threadIdx.x == 0) {
    if (dg) dg[0] = clock64();
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < FA_NS; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&pv_done[s], 1);
      mbar_init(&p_full[s], FA_SOFT);
    }
    for (int qd = 0; qd < 4; ++qd) mbar_init(&xbar[qd], 64);
    *abort_flag = 0;
    fence_barrier_init();
    // the Q tile depends on nothing below: start its load now, so its latency
    // runs under the tile-list scan and the TMEM allocation
    prefetch_tmap(&tmQ);
    mbar_arrive_expect_tx(q_full, TILE_BYTES);
    tma_load_2d(smem + OFF_Q, &tmQ, q_full, h * FB, q0);
    tma_load_2d(smem + OFF_Q + CHUNK_BYTES, &tmQ, q_full, h * FB + 64, q0);
  }
  // visible key tiles of this query block, computed once (entries: kt | TILE_FULL)
  int* tlist = reinterpret_cast<int*>(smem + OFF_TL);
  int* tcount = tlist + MAX_KT;
  if (warp == 0) {
    // sliding window: smallest position among this block's queries
    int qpmin = 0x7fffffff;
    if (p.window > 0) {
      for (int r = lane; r < FB; r += 32)
        if (g0 + r <= g_last) qpmin = min(qpmin, __ldg(p.pos + g0 + r));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) qpmin = min(qpmin, __shfl_xor_sync(0xffffffffu, qpmin, o));
    }
    int count = 0;
    for (int base = 0; base <= kt_last; base += 32) {
      const int kt = base + lane;
      bool vis = kt <= kt_last && tile_visible(p, kt, g0);
      if (vis && p.window > 0) vis = qpmin - __ldg(p.tile_pmax + kt) < p.window;
      const bool full = vis && p.window <= 0 && tile_full(p, kt, g0, g_last);
      const unsigned m = __ballot_sync(0xffffffffu, vis);
      const int pos = count + __popc(m & ((1u << lane) - 1u));
      if (vis && pos < MAX_KT) tlist[pos] = kt | (full ? TILE_FULL : 0);
      count += __popc(m);
    }
    if (lane == 0) *tcount = min(count, MAX_KT);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_o = tmem + FA_NS * FB;
  const int ntl = *tcount;
  if (dg && threadIdx.x == 64) {
    dg[1] = clock64();
    dg[36] = ntl;
  }

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      long long wke = 0, wve = 0;
      // K runs one tile ahead of V: K(0), K(1), V(0), K(2), V(1), ...  The
      // S of tile n+2 is issued once P V of tile n-1 completes, and its K
      // load must not queue behind the V load that waits for that P V
      auto load_k = [&](int n) -> bool {
        const int s = n & 1, kt = tlist[n] & (TILE_FULL - 1);
        const long long c0 = tick();
        if (!mbar_wait(&k_empty[s], ((n >> 1) & 1) ^ 1, abort_flag, p.err, 11)) return false;
        wke += tick() - c0;
        uint8_t* kb = smem + OFF_K + s * TILE_BYTES;
        mbar_arrive_expect_tx(&k_full[s], TILE_BYTES);
        tma_load_2d(kb, &tmK, &k_full[s], hk * FB, kt * FB);
        tma_load_2d(kb + CHUNK_BYTES, &tmK, &k_full[s], hk * FB + 64, kt * FB);
        return true;
      };
      auto load_v = [&](int n) -> bool {
        const int s = n & 1, kt = tlist[n] & (TILE_FULL - 1);
        const long long c0 = tick();
        if (!mbar_wait(&v_empty[s], ((n >> 1) & 1) ^ 1, abort_flag, p.err, 19)) return false;
        wve += tick() - c0;
        uint8_t* vb = smem + OFF_V + s * TILE_BYTES;
        mbar_arrive_expect_tx(&v_full[s], TILE_BYTES);
        tma_load_2d(vb, &tmV, &v_full[s], hk * FB, kt * FB);
        tma_load_2d(vb + CHUNK_BYTES, &tmV, &v_full[s], hk * FB + 64, kt * FB);
        return true;
      };
      bool ok = ntl == 0 || load_k(0);
      if (ok && ntl > 1) ok = load_k(1);
      for (int n = 0; ok && n < ntl; ++n) {
        ok = load_v(n);
        if (ok && n + 2 < ntl) ok = load_k(n + 2);
      }
      if (dg) {
        dg[44] = wke;
        dg[45] = wve;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16(FB, FB);
      constexpr uint32_t idO = idesc_bf16_bmn(FB, FB);
      const uint32_t qa = smem_addr(smem + OFF_Q);
      long long c0 = tick();
      bool ok = mbar_wait(q_full, 0, abort_flag, p.err, 12);
      long long wq = tick() - c0, wk = 0, ws = 0, wp = 0, wv = 0, is = 0, ipv = 0;
      tc_fence_after();
      auto issue_pv = [&](int n) -> bool {  // O += P_n V_n, P_n read from TMEM (S buffer n%3)
        const int s = n & 1, b = n % FA_NS;
        long long c1 = tick();
        if (!mbar_wait(&p_full[b], (n / FA_NS) & 1, abort_flag, p.err, 13)) return false;
        wp += tick() - c1;
        c1 = tick();
        if (!mbar_wait(&v_full[s], (n >> 1) & 1, abort_flag, p.err, 10)) return false;
        wv += tick() - c1;
        tc_fence_after();
        const uint32_t va = smem_addr(smem + OFF_V + s * TILE_BYTES);
        const uint32_t pt = tmem + b * FB;  // each half's P in the first 32 columns of its S columns
        c1 = tick();
#pragma unroll
        for (int kk = 0; kk < FB / 16; ++kk)
          mma_bf16_ts(tmem_o, pt + (kk >> 2) * 64 + (kk & 3) * 8, desc_mn_sw128(va + kk * 2048, CHUNK_BYTES), idO,
                      (n > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&v_empty[s]);
        mma_commit(&pv_done[b]);
        if (dg) {
          const long long c2 = clock64();
          ipv += c2 - c1;
          if (n < 16) dg[64 + n] = c2;
        }
        return true;
      };
      // S(0), S(1), then per tile n: S(n+2) (into the buffer of tile n-1,
      // whose P V was issued just before) and P V(n) (after the softmax of
      // tile n), so the scores run two tiles ahead of the softmax
      auto issue_s = [&](int n) -> bool {
        const int s = n & 1, b = n % FA_NS;
        long long c1 = tick();
        if (!mbar_wait(&k_full[s], (n >> 1) & 1, abort_flag, p.err, 14)) return false;
        wk += tick() - c1;
        // no wait for the buffer: its last reader, P V of tile n-3, was
        // issued before by this thread, and tcgen05.mma operations issued by
        // one thread execute in issue order
        if (dg && n == 0) dg[42] = clock64();
        tc_fence_after();
        const uint32_t ka = smem_addr(smem + OFF_K + s * TILE_BYTES);
        c1 = tick();
#pragma unroll
        for (int kk = 0; kk < FB / 16; ++kk)
          mma_bf16(tmem + b * FB, desc_k_sw128(qa + (kk >> 2) * CHUNK_BYTES + (kk & 3) * 32),
                   desc_k_sw128(ka + (kk >> 2) * CHUNK_BYTES + (kk & 3) * 32), idS, kk > 0 ? 1u : 0u);
        mma_commit(&s_full[b]);
        mma_commit(&k_empty[s]);
        if (dg) {
          const long long c2 = clock64();
          is += c2 - c1;
          if (n < 16) dg[48 + n] = c2;
        }
        return true;
      };
      if (ok && ntl > 0) ok = issue_s(0);
      if (ok && ntl > 1) ok = issue_s(1);
      for (int n = 0; ok && n < ntl; ++n) {
        if (n + 2 < ntl) ok = issue_s(n + 2);
        if (ok) ok = issue_pv(n);
      }
      if (dg) {
        dg[37] = wk;
        dg[38] = ws;
        dg[39] = wp;
        dg[40] = wv;
        dg[41] = wq;
        dg[43] = clock64();
        dg[80] = is;
        dg[81] = ipv;
      }
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int quad = warp & 3;         // TMEM lane quadrant this warp may access
    const int half = (warp - 2) >> 2;  // key columns (S) and output columns (O) [64*half, 64*half+64)
    const int row = quad * 32 + lane;
    const int gi = g0 + row;  // global query position of this thread's row
    const int pos_i = (p.window > 0 && gi < p.Tk) ? __ldg(p.pos + gi) : 0;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    float* xch = reinterpret_cast<float*>(smem + OFF_X);  // [slot][half][row]; slots 0/1 max, 2 sum
    float m_ref = -INFINITY, l = 0.f;  // l: this half's share of the row sum
    int* ke_w = reinterpret_cast<int*>(smem + OFF_KE) + (warp - 2) * 64;
    int n = 0;
    bool ok = true;
    for (; n < ntl; ++n) {
      const int kt = tlist[n] & (TILE_FULL - 1);
      const bool full_tile = (tlist[n] & TILE_FULL) != 0;
      const int b = n % FA_NS, par = n & 1;
      const int k0 = kt * FB + half * 64;
      // a partially visible tile needs kend of the warp's 64 keys: each lane
      // loads two before the wait for S (the load latency runs under it) and
      // the warp shares them through its shared-memory slot afterwards
      int2 kev = make_int2(0, 0);
      if (!full_tile) {
        const int j = k0 + 2 * lane;
        if (j + 1 < p.Tk) kev = __ldg(reinterpret_cast<const int2*>(p.kend + j));
        else if (j < p.Tk) kev.x = __ldg(p.kend + j);
      }
      if (!mbar_wait_warp(&s_full[b], (n / FA_NS) & 1, abort_flag, p.err, 16)) { ok = false; break; }
      if (dg && threadIdx.x == 64 && n < 16) dg[2 + 2 * n] = clock64();
      if (!full_tile) {
        __syncwarp();  // the previous partial tile's reads are done
        reinterpret_cast<int2*>(ke_w)[lane] = kev;
        __syncwarp();
      }
      tc_fence_after();
      float sv[64];
      {
        uint32_t r[2][32];
#pragma unroll
        for (int c = 0; c < 2; ++c) tmem_ld32(tmem + lane_base + b * FB + half * 64 + c * 32, r[c]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e) sv[c * 32 + e] = __uint_as_float(r[c][e]);
      }
      // mask and running max on the raw scores (the scale is positive, so it
      // is applied once to the max and folded into the exponent's FMA below);
      // four independent max chains instead of one 64-long dependency chain
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      if (full_tile) {
#pragma unroll
        for (int c = 0; c < 64; ++c) mx4[c & 3] = fmaxf(mx4[c & 3], sv[c]);
      } else {
#pragma unroll
        for (int c = 0; c < 64; c += 4) {
          const int4 ke = reinterpret_cast<const int4*>(ke_w)[c / 4];  // keys past Tk hold 0: not visible
          const int kv[4] = {ke.x, ke.y, ke.z, ke.w};
          int pj[4] = {0, 0, 0, 0};
          if (p.window > 0) {
#pragma unroll
            for (int e = 0; e < 4; ++e) pj[e] = k0 + c + e < p.Tk ? __ldg(p.pos + k0 + c + e) : 0;
          }
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = k0 + c + e;
            const bool vis = (j <= gi) && (gi < kv[e]) && (p.window <= 0 || pos_i - pj[e] < p.window);
            const float x = vis ? sv[c + e] : -INFINITY;
            sv[c + e] = x;
            mx4[e] = fmaxf(mx4[e], x);
          }
        }
      }
      float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * p.scale_log2;
      // row max over both halves (bounded mbarrier exchange between the two warps)
      xch[(par * 2 + half) * FB + row] = mx;
      mbar_arrive(&xbar[quad]);
      if (!mbar_wait_warp(&xbar[quad], n & 1, abort_flag, p.err, 19)) { ok = false; break; }
      mx = fmaxf(mx, xch[(par * 2 + (half ^ 1)) * FB + row]);
      // lazy rescale: a row moves its reference max only when the tile max
      // exceeds it by more than 2^8 (both halves decide alike: same max).
      // tcgen05.ld/st are warp-collective, so the warp rescales its O columns
      // when any of its rows needs it (alpha = 1 for the others).  Only then
      // does it wait for P V of the previous tile (O is being accumulated);
      // otherwise the softmax runs ahead of the P V MMAs.  The wait stays
      // within one phase: s_full of this tile already implies P V of tile
      // n-3 completed (both were committed by the MMA thread in order), and
      // tile n-4 was the previous user of the barrier.
      const bool move = mx > m_ref + kRescaleThreshold || (m_ref == -INFINITY && mx > -INFINITY);
      const bool scale_o = move && n > 0 && m_ref > -INFINITY;
      if (__any_sync(0xffffffffu, scale_o)) {
        if (!mbar_wait_warp(&pv_done[(n - 1) % FA_NS], ((n - 1) / FA_NS) & 1, abort_flag, p.err, 17)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float alpha = scale_o ? exp2f(m_ref - mx) : 1.f;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem_o + lane_base + half * 64 + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
          tmem_st32(tmem_o + lane_base + half * 64 + c * 32, r);
        }
        tmem_wait_st();
        l *= alpha;
      }
      if (move) m_ref = mx;
      // P = exp2(s - m_ref) as bf16 into tensor memory: this half's 64 keys
      // as 32 columns of bf16 pairs over the first half of its own S columns
      // (the P V MMA reads its A operand there)
      // exponent = s * scale_log2 - m_ref in one FMA; a masked score (-inf)
      // gives exp2(-inf) = 0, and a row with no visible key yet (m_ref =
      // -inf) subtracts 0 instead.  One pair in kExp2PolyEvery goes through
      // the polynomial exp2 on the FMA pipe instead of the MUFU pipe, whose
      // 16 results per clock per SM would otherwise bound the softmax.
      const float nm = m_ref == -INFINITY ? 0.f : -m_ref;
      float rs4[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t pk[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const float x0 = fmaf(sv[2 * c], p.scale_log2, nm), x1 = fmaf(sv[2 * c + 1], p.scale_log2, nm);
        float e0, e1;
        if (c % kExp2PolyEvery == kExp2PolyEvery - 1) {
          e0 = exp2_poly(x0);
          e1 = exp2_poly(x1);
        } else {
          e0 = exp2f(x0);
          e1 = exp2f(x1);
        }
        rs4[c & 3] += e0 + e1;
        pk[c] = pack_bf16x2(e0, e1);
      }
      tmem_st32(tmem + lane_base + b * FB + half * 64, pk);
      tmem_wait_st();
      l += (rs4[0] + rs4[1]) + (rs4[2] + rs4[3]);
      tc_fence_before();
      mbar_arrive(&p_full[b]);
      if (dg && threadIdx.x == 64 && n < 16) dg[3 + 2 * n] = clock64();
    }
    if (dg && threadIdx.x == 64) dg[34] = clock64();
    // epilogue: O / l and the LSE (the two halves' sums are exchanged once more)
    const int qrow = q0 + row;
    if (ok && n > 0) {
      xch[(4 + half) * FB + row] = l;  // own slot: the max slots may still be read by the partner
      bool got = false;
      if (mbar_wait_warp(&pv_done[(n - 1) % FA_NS], ((n - 1) / FA_NS) & 1, abort_flag, p.err, 18)) {
        mbar_arrive(&xbar[quad]);
        got = mbar_wait_warp(&xbar[quad], n & 1, abort_flag, p.err, 20);
      }
      if (got) {
        tc_fence_after();
        l += xch[(4 + (half ^ 1)) * FB + row];
        // a sink adds exp(sink) to the denominator (log2 units relative to m_ref)
        if (p.sinks && m_ref > -INFINITY) l += exp2f(__ldg(p.sinks + h) * kLog2eF - m_ref);
        const float inv = l > 0.f ? 1.f / l : 0.f;
        // the warp's 32 rows x 64 columns (128 bytes a row) go out through a
        // per-warp block of the (now unused) P region, 16-byte chunks XOR-
        // swizzled by row: each store instruction then writes 4 rows x 128
        // contiguous bytes instead of 32 rows x 16 bytes
        uint8_t* stg = smem + OFF_P + (warp - 2) * 32 * 128;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem_o + lane_base + half * 64 + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            uint4 o;
            o.x = pack_bf16x2(__uint_as_float(r[j + 0]) * inv, __uint_as_float(r[j + 1]) * inv);
            o.y = pack_bf16x2(__uint_as_float(r[j + 2]) * inv, __uint_as_float(r[j + 3]) * inv);
            o.z = pack_bf16x2(__uint_as_float(r[j + 4]) * inv, __uint_as_float(r[j + 5]) * inv);
            o.w = pack_bf16x2(__uint_as_float(r[j + 6]) * inv, __uint_as_float(r[j + 7]) * inv);
            const int u = c * 4 + j / 8;  // 16-byte chunk of the 128-byte row
            *reinterpret_cast<uint4*>(stg + lane * 128 + ((u ^ (lane & 7)) << 4)) = o;
          }
        }
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int rr = 4 * k + (lane >> 3), u = lane & 7;
          const int orow = q0 + quad * 32 + rr;
          const uint4 o = *reinterpret_cast<const uint4*>(stg + rr * 128 + ((u ^ (rr & 7)) << 4));
          if (orow < p.Tq)
            *reinterpret_cast<uint4*>(p.o + (int64_t)orow * p.ldo + (int64_t)h * FB + half * 64 + u * 8) = o;
        }
        if (qrow < p.Tq && half == 0)
          p.lse[(int64_t)h * p.Tq + qrow] =
              l > 0.f ? (m_ref + log2f(l)) / kLog2eF : (p.sinks ? __ldg(p.sinks + h) : -INFINITY);
      }
    } else if (ok && qrow < p.Tq) {  // no visible key
      __nv_bfloat16* dst = p.o + (int64_t)qrow * p.ldo + (int64_t)h * FB + half * 64;
      for (int j = 0; j < 64; j += 8) *reinterpret_cast<uint4*>(dst + j) = make_uint4(0, 0, 0, 0);
      if (half == 0) p.lse[(int64_t)h * p.Tq + qrow] = p.sinks ? __ldg(p.sinks + h) : -INFINITY;
    }
    if (dg && threadIdx.x == 64) dg[35] = clock64();
  }
  tc_fence_before();
  __syncthreads();
  if (dg && threadIdx.x == 0) dg[46] = clock64();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// q [Tq, Hq, 128] (rows at global positions q_off + row), k/v [Tk, Hkv, 128];
// heads packed, rows 16-byte aligned.  Returns {o [Tq, Hq, 128] bf16, lse [Hq, Tq] fp32}.
std::vector<torch::Tensor> attn_fwd_tc(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor kend,
                                       torch::Tensor tile_kmax, torch::Tensor tile_kmin, double scale, int64_t q_off,
                                       c10::optional<torch::Tensor> pos, c10::optional<torch::Tensor> tile_pmax,
                                       int64_t window, c10::optional<torch::Tensor> sinks,
                                       c10::optional<torch::Tensor> diag) {
  const int64_t Tq = q.size(0), Hq = q.size(1), D = q.size(2), Tk = k.size(0), Hkv = k.size(1);
  TORCH_CHECK(D == 128, "attention kernel supports head_dim 128");
  TORCH_CHECK(Hq % Hkv == 0, "GQA: q heads must be a multiple of kv heads");
  TORCH_CHECK(q_off >= 0 && q_off + Tq <= Tk, "query range must lie inside the key range");
  for (auto* t : {&q, &k, &v}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->dim() == 3, "bf16 CUDA [T, H, 128]");
    TORCH_CHECK(t->stride(2) == 1 && t->stride(1) == 128, "heads must be packed");
    TORCH_CHECK(t->stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(t->data_ptr()) % 16) == 0,
                "rows must be 16-byte aligned");
  }
  TORCH_CHECK(v.size(0) == Tk && v.size(1) == Hkv, "v shape");
  TORCH_CHECK(kend.scalar_type() == at::kInt && kend.numel() == Tk && kend.is_contiguous());
  TORCH_CHECK((reinterpret_cast<uintptr_t>(kend.data_ptr()) % 16) == 0, "kend must be 16-byte aligned");
  TORCH_CHECK(tile_kmax.scalar_type() == at::kInt && tile_kmax.numel() >= (Tk + 63) / 64);
  TORCH_CHECK(tile_kmin.scalar_type() == at::kInt && tile_kmin.numel() >= (Tk + 63) / 64);
  TORCH_CHECK((Tk + FB - 1) / FB <= MAX_KT, "attention rows longer than ", MAX_KT * FB, " keys");
  auto o = torch::empty({Tq, Hq, D}, q.options());
  auto lse = torch::empty({Hq, Tq}, q.options().dtype(at::kFloat));
  if (Tq == 0) return {o, lse};
  // 2-D views [rows, heads*128] for the tensor maps
  auto q2 = q.as_strided({Tq, Hq * D}, {q.stride(0), 1});
  auto k2 = k.as_strided({Tk, Hkv * D}, {k.stride(0), 1});
  auto v2 = v.as_strided({Tk, Hkv * D}, {v.stride(0), 1});
  const CUtensorMap mq = make_tmap_bf16(q2, FB), mk = make_tmap_bf16(k2, FB), mv = make_tmap_bf16(v2, FB);
  int dev = 0;
  ART_CUDA_CHECK(cudaGetDevice(&dev));
  FaArgs a;
  a.kend = kend.data_ptr<int>();
  a.tile_kmax = tile_kmax.data_ptr<int>();
  a.tile_kmin = tile_kmin.data_ptr<int>();
  a.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  a.ldo = o.stride(0);
  a.lse = lse.data_ptr<float>();
  a.Tq = (int)Tq;
  a.Tk = (int)Tk;
  a.q_off = (int)q_off;
  a.Hq = (int)Hq;
  a.Hkv = (int)Hkv;
  a.scale_log2 = (float)(scale * kLog2eF);
  a.err = tc_error_ptr(dev);
  a.window = window > 0 ? (int)window : 0;
  a.pos = nullptr;
  a.tile_pmax = nullptr;
  if (a.window) {
    TORCH_CHECK(pos.has_value() && tile_pmax.has_value(), "a sliding window needs positions and tile position maxima");
    TORCH_CHECK(pos->is_cuda() && pos->scalar_type() == at::kInt && pos->is_contiguous() && pos->numel() == Tk);
    TORCH_CHECK(tile_pmax->is_cuda() && tile_pmax->scalar_type() == at::kInt && tile_pmax->is_contiguous() &&
                tile_pmax->numel() >= (Tk + FB - 1) / FB);
    TORCH_CHECK((reinterpret_cast<uintptr_t>(pos->data_ptr()) % 16) == 0, "positions must be 16-byte aligned");
    a.pos = pos->data_ptr<int>();
    a.tile_pmax = tile_pmax->data_ptr<int>();
  }
  a.sinks = nullptr;
  if (sinks.has_value()) {
    TORCH_CHECK(sinks->is_cuda() && sinks->scalar_type() == at::kFloat && sinks->is_contiguous() &&
                sinks->numel() == Hq, "sinks: fp32 [Hq]");
    a.sinks = sinks->data_ptr<float>();
  }
  a.diag = nullptr;
  if (diag.has_value()) {
    TORCH_CHECK(diag->is_cuda() && diag->scalar_type() == at::kLong && diag->is_contiguous() &&
                diag->numel() >= ((Tq + FB - 1) / FB) * Hq * kFaDiag, "diag: int64 [ctas, ", kFaDiag, "]");
    a.diag = reinterpret_cast<long long*>(diag->data_ptr<int64_t>());
  }
  static bool attr = false;
  if (!attr) {
    const auto smem_attr = cudaFuncAttributeMaxDynamicSharedMemorySize;
    ART_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_tc_kernel<false>, smem_attr, FA_SMEM));
    ART_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_tc_kernel<true>, smem_attr, FA_SMEM));
    attr = true;
  }
  dim3 grid((unsigned)((Tq + FB - 1) / FB), (unsigned)Hq);
  if (a.diag)
    attn_fwd_tc_kernel<true><<<grid, FA_THREADS, FA_SMEM, at::cuda::getCurrentCUDAStream()>>>(mq, mk, mv, a);
  else
    attn_fwd_tc_kernel<false><<<grid, FA_THREADS, FA_SMEM, at::cuda::getCurrentCUDAStream()>>>(mq, mk, mv, a);
  ART_CUDA_CHECK(cudaGetLastError());
  return {o, lse};
}


// ============================================================================
// Backward on the tensor cores.
//
// CTA = one work unit (128-key block kb, local 128-query tiles [t_lo, t_hi))
// x one kv head; it loops over the G q heads of that kv head and the query
// tiles, with K and V of the block resident in shared memory:
//   S^T  = K Q^T          (TMEM cols   0..127, lanes = keys)
//   dP^T = V dO^T         (TMEM cols 128..255)
//   softmax warps: P^T = exp2(S^T*scale*log2e - lse*log2e) under the mask,
//                  dS^T = P^T (dP^T - delta); dS^T as a bf16 tile in shared
//                  memory, P^T as bf16 pairs in TMEM over the dP^T columns
//                  each warp has already read (cols 128+64h .. +32)
//   dV  += P^T dO         (TMEM cols 256..383, P^T a tensor-memory A operand,
//                          dO an MN-major B operand)
//   dK  += dS^T Q         (TMEM cols 384..511)
//   dQ   = dS K           (TMEM cols 0..127, dS^T read as an MN-major A
//                          operand, K as an MN-major B operand; lanes = queries)
// then dQ*scale is added to global memory (red.global.add.v4.f32, transposed
// through a per-warp shared-memory block so each instruction writes whole
// 128-byte row segments) and, after
// the last tile, dK*scale and dV are added for the block (several units may
// share a key block).  delta = rowsum(dO * O) comes from attn_bwd_delta.
// ============================================================================

namespace {

constexpr int QDO_ST = 1;  // Q / dO stages (shared memory goes to the dQ staging below)
constexpr int B_OFF_K = 0;
constexpr int B_OFF_V = TILE_BYTES;
constexpr int B_OFF_Q = 2 * TILE_BYTES;
constexpr int B_OFF_DO = B_OFF_Q + QDO_ST * TILE_BYTES;
constexpr int B_OFF_DS = B_OFF_DO + QDO_ST * TILE_BYTES;
// per softmax warp a 32 x 32 fp32 block in the 128-byte-swizzled layout of a
// TMA box (the source of the dQ / dK / dV reduce-adds); 1024-byte aligned
constexpr int B_OFF_DQ = B_OFF_DS + TILE_BYTES;
constexpr int B_STG = 32 * 32 * 4;
// per softmax warp: log2-scaled LSE, delta and (sliding window) positions of
// its 64 query columns of the current tile
constexpr int B_OFF_LD = B_OFF_DQ + 8 * B_STG;
constexpr int B_OFF_BAR = B_OFF_LD + 8 * 3 * 64 * 4;
constexpr int FB_SMEM = B_OFF_BAR + 256 + 1024;
// 2 control warps + 8 softmax warps: two warps per TMEM lane quadrant, each
// taking 64 of the 128 query columns (the backward needs no row reduction)
constexpr int FB_THREADS = 320;
constexpr int FB_SOFT = 256;

struct FbArgs {
  const int* kend;
  const int* units;  // [n, 3]
  const float* lse;    // [Hq, Tq] natural log
  const float* delta;  // [Hq, Tq]
  float* dq;           // [Tq, Hq, 128]
  float* dk;           // [Tk, Hkv, 128]
  float* dv;
  int Tq, Tk, q_off, Hq, Hkv;
  float scale, scale_log2;
  int* err;
  const int* pos;  // [Tk] token positions (sliding window only)
  int window;      // > 0: also pos[query] - pos[key] < window
  long long* diag;  // phase clocks per CTA (diag build only), kFbDiag int64 slots each
};
constexpr int kFbDiag = 128;


}  // namespace

__global__ void attn_bwd_delta_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ o,
                                      int64_t ldo, float* __restrict__ delta, int Tq, int Hq) {
  const int w = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (w >= Tq * Hq) return;
  const int t = w / Hq, h = w % Hq;
  const uint2 a = *reinterpret_cast<const uint2*>(dout + ((int64_t)t * Hq + h) * FB + lane * 4);
  const uint2 b = *reinterpret_cast<const uint2*>(o + (int64_t)t * ldo + (int64_t)h * FB + lane * 4);
  const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(&a);
  const __nv_bfloat16* y = reinterpret_cast<const __nv_bfloat16*>(&b);
  float s = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) s += bf2f(x[e]) * bf2f(y[e]);
  s = warp_sum(s);
  if (lane == 0) delta[(int64_t)h * Tq + t] = s;
}

// DIAG: the phase-clock build (FbArgs::diag), kept out of the production instance
template <bool DIAG>
__global__ void __launch_bounds__(FB_THREADS, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                       const __grid_constant__ CUtensorMap tmDQ, const __grid_constant__ CUtensorMap tmDK,
                       const __grid_constant__ CUtensorMap tmDV, const FbArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + B_OFF_BAR);
  uint64_t* kv_full = bars + 0;
  uint64_t* sdp_full = bars + 1;
  uint64_t* ds_full = bars + 2;
  uint64_t* dq_full = bars + 3;
  uint64_t* dq_free = bars + 4;
  uint64_t* qdo_full = bars + 5;   // [2]
  uint64_t* qdo_empty = bars + 7;  // [2]
  uint64_t* dv_done = bars + 9;    // dV / dK of a tile finished (P^T read from the dP^T columns)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kb = p.units[blockIdx.x * 3 + 0];
  const int t_lo = p.units[blockIdx.x * 3 + 1], t_hi = p.units[blockIdx.x * 3 + 2];
  const int hk = blockIdx.y;
  const int G = p.Hq / p.Hkv;
  const int ntiles = t_hi - t_lo;
  const int iters = G * ntiles;  // iteration i: head hk*G + i / ntiles, tile t_lo + i % ntiles
  long long* dg = DIAG ? p.diag + (int64_t)(blockIdx.y * gridDim.x + blockIdx.x) * kFbDiag : nullptr;
  auto tick = [&]() -> long long { return DIAG ? (long long)clock64() : 0ll; };

  if (threadIdx.x == 0) {
    if (dg) {
      dg[0] = clock64();
      dg[2] = iters;
    }
    mbar_init(kv_full, 1);
    for (int st = 0; st < 2; ++st) {
      mbar_init(&qdo_full[st], 1);
      mbar_init(&qdo_empty[st], 1);
    }
    mbar_init(sdp_full, 1);
    mbar_init(dv_done, 1);
    mbar_init(ds_full, FB_SOFT);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, FB_SOFT);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (dg && threadIdx.x == 64) dg[1] = clock64();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      long long wqe = 0;
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      prefetch_tmap(&tmDO);
      mbar_arrive_expect_tx(kv_full, 2 * TILE_BYTES);
      tma_load_2d(smem + B_OFF_K, &tmK, kv_full, hk * FB, kb * FB);
      tma_load_2d(smem + B_OFF_K + CHUNK_BYTES, &tmK, kv_full, hk * FB + 64, kb * FB);
      tma_load_2d(smem + B_OFF_V, &tmV, kv_full, hk * FB, kb * FB);
      tma_load_2d(smem + B_OFF_V + CHUNK_BYTES, &tmV, kv_full, hk * FB + 64, kb * FB);
      for (int i = 0; i < iters; ++i) {  // Q / dO double-buffered: tile i+1 loads while tile i computes
        const int h = hk * G + i / ntiles, t = t_lo + i % ntiles;
        const int st = i % QDO_ST;
        const long long c0 = tick();
        if (!mbar_wait(&qdo_empty[st], ((i / QDO_ST) & 1) ^ 1, abort_flag, p.err, 21)) break;
        wqe += tick() - c0;
        uint8_t* qb = smem + B_OFF_Q + st * TILE_BYTES;
        uint8_t* db = smem + B_OFF_DO + st * TILE_BYTES;
        mbar_arrive_expect_tx(&qdo_full[st], 2 * TILE_BYTES);
        tma_load_2d(qb, &tmQ, &qdo_full[st], h * FB, t * FB);
        tma_load_2d(qb + CHUNK_BYTES, &tmQ, &qdo_full[st], h * FB + 64, t * FB);
        tma_load_2d(db, &tmDO, &qdo_full[st], h * FB, t * FB);
        tma_load_2d(db + CHUNK_BYTES, &tmDO, &qdo_full[st], h * FB + 64, t * FB);
      }
      if (dg) dg[78] = wqe;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idKK = idesc_bf16(FB, FB);                  // both K-major
      constexpr uint32_t idKM = idesc_bf16_bmn(FB, FB);              // B MN-major
      constexpr uint32_t idMM = idesc_bf16_bmn(FB, FB) | (1u << 15);  // A and B MN-major
      const uint32_t ka = smem_addr(smem + B_OFF_K), va = smem_addr(smem + B_OFF_V);
      const uint32_t dsa = smem_addr(smem + B_OFF_DS);
      long long w_q = 0, w_dv = 0, i_dp = 0, w_dq = 0, i_s = 0, w_ds = 0, i_dvdk = 0, i_dq = 0, c0 = 0;
      if (mbar_wait(kv_full, 0, abort_flag, p.err, 22)) {
        for (int i = 0; i < iters; ++i) {
          const int st = i % QDO_ST;
          const uint32_t qa = smem_addr(smem + B_OFF_Q + st * TILE_BYTES);
          const uint32_t doa = smem_addr(smem + B_OFF_DO + st * TILE_BYTES);
          c0 = tick();
          if (!mbar_wait(&qdo_full[st], (i / QDO_ST) & 1, abort_flag, p.err, 23)) break;
          w_q += tick() - c0;
          // dP^T = V dO^T first: its columns (128..255) only have to be free of
          // the previous tile's P^T, i.e. its dV MMA done; it then runs while
          // the softmax warps still read the previous dQ out of columns 0..127
          c0 = tick();
          if (i > 0 && !mbar_wait(dv_done, (i - 1) & 1, abort_flag, p.err, 28)) break;
          w_dv += tick() - c0;
          tc_fence_after();
          c0 = tick();
#pragma unroll
          for (int kk = 0; kk < FB / 16; ++kk) {
            const uint32_t ko = (kk >> 2) * CHUNK_BYTES + (kk & 3) * 32;
            mma_bf16(tmem + 128, desc_k_sw128(va + ko), desc_k_sw128(doa + ko), idKK, kk > 0 ? 1u : 0u);
          }
          i_dp += tick() - c0;
          c0 = tick();
          if (!mbar_wait(dq_free, (i & 1) ^ 1, abort_flag, p.err, 24)) break;
          w_dq += tick() - c0;
          tc_fence_after();
          c0 = tick();
#pragma unroll
          for (int kk = 0; kk < FB / 16; ++kk) {
            const uint32_t ko = (kk >> 2) * CHUNK_BYTES + (kk & 3) * 32;
            mma_bf16(tmem + 0, desc_k_sw128(ka + ko), desc_k_sw128(qa + ko), idKK, kk > 0 ? 1u : 0u);
          }
          mma_commit(sdp_full);
          i_s += tick() - c0;
          c0 = tick();
          if (!mbar_wait(ds_full, i & 1, abort_flag, p.err, 25)) break;
          w_ds += tick() - c0;
          tc_fence_after();
          c0 = tick();
#pragma unroll
          for (int kk = 0; kk < FB / 16; ++kk) {
            const uint32_t ko = (kk >> 2) * CHUNK_BYTES + (kk & 3) * 32;
            const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
            // dV += P^T dO with P^T read from TMEM (bf16 pairs over the dP^T columns: queries
            // [64h, 64h+64) at columns 128 + 64h .. +32)
            mma_bf16_ts(tmem + 256, tmem + 128 + (kk >> 2) * 64 + (kk & 3) * 8,
                        desc_mn_sw128(doa + kk * 2048, CHUNK_BYTES), idKM, acc);
            mma_bf16(tmem + 384, desc_k_sw128(dsa + ko), desc_mn_sw128(qa + kk * 2048, CHUNK_BYTES), idKM, acc);
          }
          mma_commit(&qdo_empty[st]);
          mma_commit(dv_done);
          i_dvdk += tick() - c0;
          c0 = tick();
#pragma unroll
          for (int kk = 0; kk < FB / 16; ++kk)
            mma_bf16(tmem + 0, desc_mn_sw128(dsa + kk * 2048, CHUNK_BYTES),
                     desc_mn_sw128(ka + kk * 2048, CHUNK_BYTES), idMM, kk > 0 ? 1u : 0u);
          mma_commit(dq_full);
          i_dq += tick() - c0;
        }
      }
      if (dg) {
        dg[70] = w_q;
        dg[71] = w_dv;
        dg[72] = i_dp;
        dg[73] = w_dq;
        dg[74] = i_s;
        dg[75] = w_ds;
        dg[76] = i_dvdk;
        dg[77] = i_dq;
      }
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogues
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;  // query / head-dim columns [64*half, 64*half + 64)
    const int row = quad * 32 + lane;  // TMEM lane: key row (S^T, dP^T, dK, dV) or query row (dQ)
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const int j = kb * FB + row;  // this thread's key
    const int kend_j = j < p.Tk ? __ldg(p.kend + j) : 0;
    const int pos_j = (p.window > 0 && j < p.Tk) ? __ldg(p.pos + j) : 0;
    const int sw = row & 7;
    // the warp's 32 keys: a 32-query chunk is fully visible to all of them
    // when it lies at or after the last key and before the smallest kend
    int kmin_w = j < p.Tk ? kend_j : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) kmin_w = min(kmin_w, __shfl_xor_sync(0xffffffffu, kmin_w, o));
    const int jmax_w = kb * FB + quad * 32 + 31;
    float* lsw = reinterpret_cast<float*>(smem + B_OFF_LD) + (warp - 2) * 3 * 64;  // [lse2 64][delta 64][pos 64]
    int* psw = reinterpret_cast<int*>(lsw + 128);
    uint8_t* stg = smem + B_OFF_DQ + (warp - 2) * B_STG;
    // the warp's own rows of the dS tile: 32 keys x 64 queries = 4 KB, 1024-byte aligned
    uint8_t* stg2 = smem + B_OFF_DS + half * CHUNK_BYTES + quad * 32 * 128;
    bool ok = true;
    for (int i = 0; i < iters && ok; ++i) {
      const int h = hk * G + i / ntiles, t = t_lo + i % ntiles;
      // lane e fetches the LSE / delta of query columns 64*half + e and +32,
      // issued before the MMA wait so the loads overlap it
      const float* lse_h = p.lse + (int64_t)h * p.Tq;
      const float* del_h = p.delta + (int64_t)h * p.Tq;
      float lse_pf[2], del_pf[2];
      int pos_pf[2] = {0, 0};
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int ql_mine = t * FB + (2 * half + cc) * 32 + lane;
        lse_pf[cc] = ql_mine < p.Tq ? __ldg(lse_h + ql_mine) * kLog2eF : INFINITY;
        del_pf[cc] = ql_mine < p.Tq ? __ldg(del_h + ql_mine) : 0.f;
        if (p.window > 0) pos_pf[cc] = ql_mine < p.Tq ? __ldg(p.pos + p.q_off + ql_mine) : 0;
      }
      if (!mbar_wait_warp(sdp_full, i & 1, abort_flag, p.err, 26)) { ok = false; break; }
      if (dg && threadIdx.x == 64 && i < 16) dg[4 + 4 * i] = clock64();
      // shared with the whole warp through its slot (broadcast reads below
      // instead of three shuffles per element)
      __syncwarp();
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        lsw[cc * 32 + lane] = lse_pf[cc];
        lsw[64 + cc * 32 + lane] = del_pf[cc];
        psw[cc * 32 + lane] = pos_pf[cc];
      }
      __syncwarp();
      tc_fence_after();
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int c = 2 * half + cc;
        uint32_t rs[32], rd[32];
        uint32_t pp[16];  // P^T of these 32 queries, bf16 pairs
        tmem_ld32(tmem + lane_base + c * 32, rs);
        tmem_ld32(tmem + lane_base + 128 + c * 32, rd);
        const int q0c = t * FB + c * 32;  // local query of the chunk's first column
        const bool full = p.window <= 0 && jmax_w <= p.q_off + q0c && kmin_w > p.q_off + q0c + 31 &&
                          q0c + 31 < p.Tq;
        tmem_wait_ld();
        if (dg && threadIdx.x == 64 && i < 8 && cc == 0) dg[80 + 2 * i] = clock64();
        uint32_t dd[16];
        // three passes over the 32 columns, each of 32 independent chains (the
        // exponentials, then dS, then the bf16 packs), so that the latencies
        // of one column's steps overlap the other columns' instead of queuing
        const float4* l4p = reinterpret_cast<const float4*>(lsw + cc * 32);
        const float4* d4p = reinterpret_cast<const float4*>(lsw + 64 + cc * 32);
        float pv[32];
#pragma unroll
        for (int e = 0; e < 32; e += 4) {
          const float4 l4 = l4p[e / 4];
          // queries past Tq carry LSE = +inf: their P is 0 on either path
          pv[e + 0] = exp2f(fmaf(__uint_as_float(rs[e + 0]), p.scale_log2, -l4.x));
          pv[e + 1] = exp2f(fmaf(__uint_as_float(rs[e + 1]), p.scale_log2, -l4.y));
          pv[e + 2] = exp2f(fmaf(__uint_as_float(rs[e + 2]), p.scale_log2, -l4.z));
          pv[e + 3] = exp2f(fmaf(__uint_as_float(rs[e + 3]), p.scale_log2, -l4.w));
        }
        if (!full) {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int qg = p.q_off + q0c + e;
            const bool vis = (j <= qg) && (qg < kend_j) && (p.window <= 0 || psw[cc * 32 + e] - pos_j < p.window);
            pv[e] = vis ? pv[e] : 0.f;
          }
        }
#pragma unroll
        for (int e = 0; e < 32; e += 4) {
          const float4 d4 = d4p[e / 4];
          rd[e + 0] = __float_as_uint(pv[e + 0] * (__uint_as_float(rd[e + 0]) - d4.x));
          rd[e + 1] = __float_as_uint(pv[e + 1] * (__uint_as_float(rd[e + 1]) - d4.y));
          rd[e + 2] = __float_as_uint(pv[e + 2] * (__uint_as_float(rd[e + 2]) - d4.z));
          rd[e + 3] = __float_as_uint(pv[e + 3] * (__uint_as_float(rd[e + 3]) - d4.w));
        }
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          pp[e] = pack_bf16x2(pv[2 * e], pv[2 * e + 1]);
          dd[e] = pack_bf16x2(__uint_as_float(rd[2 * e]), __uint_as_float(rd[2 * e + 1]));
        }
        if (dg && threadIdx.x == 64 && i < 8 && cc == 0) dg[96 + 4 * i] = clock64();
        // 32 queries = 4 units of 16 bytes of this key's row (the warp's dS
        // block doubles as dQ staging: the reduce that read it has finished)
        if (cc == 0) {
          if (lane == 0) bulk_wait_read_all();
          __syncwarp();
        }
        if (dg && threadIdx.x == 64 && i < 8 && cc == 0) dg[97 + 4 * i] = clock64();
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const int u = c * 4 + w;  // unit along the 128-query row
          const uint32_t off = (u >> 3) * CHUNK_BYTES + row * 128 + (((u & 7) ^ sw) << 4);
          *reinterpret_cast<uint4*>(smem + B_OFF_DS + off) = make_uint4(dd[4 * w], dd[4 * w + 1], dd[4 * w + 2], dd[4 * w + 3]);
        }
        // P^T of these 32 queries as 16 columns of bf16 pairs at 128 + 64*half
        // + 16*cc: over dP^T columns of queries 64*half .. +32, which this
        // warp has already read (chunk cc = 0)
        tmem_st16(tmem + lane_base + 128 + half * 64 + cc * 16, pp);
        if (dg && threadIdx.x == 64 && i < 8 && cc == 0) dg[98 + 4 * i] = clock64();
      }
      if (dg && threadIdx.x == 64 && i < 8) dg[81 + 2 * i] = clock64();
      tmem_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(ds_full);
      if (dg && threadIdx.x == 64 && i < 16) dg[5 + 4 * i] = clock64();
      // dQ tile: lanes are queries now
      if (!mbar_wait_warp(dq_full, i & 1, abort_flag, p.err, 27)) { ok = false; break; }
      if (dg && threadIdx.x == 64 && i < 16) dg[6 + 4 * i] = clock64();
      tc_fence_after();
      // both 32-column chunks of dQ into registers, then the TMEM columns are
      // released at once (the next S^T may overwrite them) and the adds go
      // out as TMA reduce-adds from the warp's swizzled staging block
      uint32_t r[2][32];
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) tmem_ld32(tmem + lane_base + (2 * half + cc) * 32, r[cc]);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(dq_free);
      // chunk 0 through the warp's staging block, chunk 1 through its 4 KB
      // block of the dS tile (free now: dq_full covered the MMAs that read
      // it; the softmax waits for this reduce's read before writing dS again)
      if (lane == 0) bulk_wait_read_all();  // the blocks' previous reduces have read them
      __syncwarp();
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        uint8_t* blk = cc ? stg2 : stg;
#pragma unroll
        for (int u = 0; u < 8; ++u)
          *reinterpret_cast<float4*>(blk + lane * 128 + ((u ^ (lane & 7)) << 4)) =
              make_float4(__uint_as_float(r[cc][4 * u]) * p.scale, __uint_as_float(r[cc][4 * u + 1]) * p.scale,
                          __uint_as_float(r[cc][4 * u + 2]) * p.scale, __uint_as_float(r[cc][4 * u + 3]) * p.scale);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_reduce_add_2d(&tmDQ, stg, h * FB + (2 * half) * 32, t * FB + quad * 32);
        tma_reduce_add_2d(&tmDQ, stg2, h * FB + (2 * half + 1) * 32, t * FB + quad * 32);
        bulk_commit_group();
      }
      if (dg && threadIdx.x == 64 && i < 16) dg[7 + 4 * i] = clock64();
    }
    if (dg && threadIdx.x == 64) dg[68] = clock64();
    // dK, dV of the block (all MMAs completed: the last dq_full covered them),
    // added with the same TMA reduce-adds; every lane runs the warp-collective
    // TMEM loads, and rows past Tk are not written by the TMA
    if (ok && iters > 0) {
#pragma unroll 1
      for (int c = 2 * half; c < 2 * half + 2; ++c) {
        uint32_t a[2][32];  // [0] dK (x scale), [1] dV: through the two staging blocks
        tmem_ld32(tmem + lane_base + 384 + c * 32, a[0]);
        tmem_ld32(tmem + lane_base + 256 + c * 32, a[1]);
        tmem_wait_ld();
        if (lane == 0) bulk_wait_read_all();
        __syncwarp();
#pragma unroll
        for (int which = 0; which < 2; ++which) {
          uint8_t* blk = which ? stg2 : stg;
          const float f = which ? 1.f : p.scale;
#pragma unroll
          for (int u = 0; u < 8; ++u)
            *reinterpret_cast<float4*>(blk + lane * 128 + ((u ^ (lane & 7)) << 4)) =
                make_float4(__uint_as_float(a[which][4 * u]) * f, __uint_as_float(a[which][4 * u + 1]) * f,
                            __uint_as_float(a[which][4 * u + 2]) * f, __uint_as_float(a[which][4 * u + 3]) * f);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_reduce_add_2d(&tmDK, stg, hk * FB + c * 32, kb * FB + quad * 32);
          tma_reduce_add_2d(&tmDV, stg2, hk * FB + c * 32, kb * FB + quad * 32);
          bulk_commit_group();
        }
      }
    }
    if (lane == 0) bulk_wait_all();  // every reduce-add has completed before the CTA exits
  }
  if (dg && threadIdx.x == 64) dg[69] = clock64();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Backward.  units [n, 3] int32 = (128-key block, first and end local
// 128-query tile).  Returns {dq [Tq,Hq,128], dk [Tk,Hkv,128], dv} fp32.
std::vector<torch::Tensor> attn_bwd_tc(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                       torch::Tensor out, torch::Tensor lse, torch::Tensor kend, torch::Tensor units,
                                       double scale, int64_t q_off, c10::optional<torch::Tensor> pos, int64_t window,
                                       c10::optional<torch::Tensor> diag) {
  const int64_t Tq = q.size(0), Hq = q.size(1), D = q.size(2), Tk = k.size(0), Hkv = k.size(1);
  TORCH_CHECK(D == 128 && Hq % Hkv == 0 && q_off >= 0 && q_off + Tq <= Tk);
  for (auto* t : {&q, &k, &v, &out}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->dim() == 3, "bf16 CUDA [T, H, 128]");
    TORCH_CHECK(t->stride(2) == 1 && t->stride(1) == 128, "heads must be packed");
    TORCH_CHECK(t->stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(t->data_ptr()) % 16) == 0,
                "rows must be 16-byte aligned");
  }
  TORCH_CHECK(dout.is_contiguous() && dout.sizes() == q.sizes() && dout.scalar_type() == at::kBFloat16);
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.is_contiguous() && lse.numel() == Hq * Tq);
  TORCH_CHECK(kend.scalar_type() == at::kInt && kend.numel() == Tk && kend.is_contiguous());
  TORCH_CHECK(units.scalar_type() == at::kInt && units.is_contiguous() && units.dim() == 2 && units.size(1) == 3);
  auto f32 = q.options().dtype(at::kFloat);
  auto dq = torch::zeros({Tq, Hq, D}, f32);
  auto dk = torch::zeros({Tk, Hkv, D}, f32);
  auto dv = torch::zeros({Tk, Hkv, D}, f32);
  const int64_t n = units.size(0);
  auto delta = torch::zeros({Hq, Tq}, f32);
  if (Tq == 0 || n == 0) return {dq, dk, dv, delta};
  auto stream = at::cuda::getCurrentCUDAStream();
  attn_bwd_delta_kernel<<<(unsigned)((Tq * Hq + 3) / 4), 128, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(out.data_ptr()),
      out.stride(0), delta.data_ptr<float>(), (int)Tq, (int)Hq);
  ART_CUDA_CHECK(cudaGetLastError());
  auto q2 = q.as_strided({Tq, Hq * D}, {q.stride(0), 1});
  auto do2 = dout.view({Tq, Hq * D});
  auto k2 = k.as_strided({Tk, Hkv * D}, {k.stride(0), 1});
  auto v2 = v.as_strided({Tk, Hkv * D}, {v.stride(0), 1});
  const CUtensorMap mq = make_tmap_bf16(q2, FB), mk = make_tmap_bf16(k2, FB), mv = make_tmap_bf16(v2, FB),
                    mdo = make_tmap_bf16(do2, FB);
  // fp32 gradients as [rows, heads*128]: targets of the TMA reduce-adds
  const CUtensorMap mdq = make_tmap_f32_32(dq.view({Tq, Hq * D})), mdk = make_tmap_f32_32(dk.view({Tk, Hkv * D})),
                    mdv = make_tmap_f32_32(dv.view({Tk, Hkv * D}));
  int dev = 0;
  ART_CUDA_CHECK(cudaGetDevice(&dev));
  FbArgs a;
  a.kend = kend.data_ptr<int>();
  a.units = units.data_ptr<int>();
  a.lse = lse.data_ptr<float>();
  a.delta = delta.data_ptr<float>();
  a.dq = dq.data_ptr<float>();
  a.dk = dk.data_ptr<float>();
  a.dv = dv.data_ptr<float>();
  a.Tq = (int)Tq;
  a.Tk = (int)Tk;
  a.q_off = (int)q_off;
  a.Hq = (int)Hq;
  a.Hkv = (int)Hkv;
  a.scale = (float)scale;
  a.scale_log2 = (float)(scale * kLog2eF);
  a.err = tc_error_ptr(dev);
  a.window = window > 0 ? (int)window : 0;
  a.pos = nullptr;
  if (a.window) {
    TORCH_CHECK(pos.has_value() && pos->is_cuda() && pos->scalar_type() == at::kInt && pos->is_contiguous() &&
                pos->numel() == Tk, "a sliding window needs int32 positions [Tk]");
    a.pos = pos->data_ptr<int>();
  }
  a.diag = nullptr;
  if (diag.has_value()) {
    TORCH_CHECK(diag->is_cuda() && diag->scalar_type() == at::kLong && diag->is_contiguous() &&
                diag->numel() >= n * Hkv * kFbDiag, "diag: int64 [units * kv heads, ", kFbDiag, "]");
    a.diag = reinterpret_cast<long long*>(diag->data_ptr<int64_t>());
  }
  static bool attr = false;
  if (!attr) {
    const auto smem_attr = cudaFuncAttributeMaxDynamicSharedMemorySize;
    ART_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_tc_kernel<false>, smem_attr, FB_SMEM));
    ART_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_tc_kernel<true>, smem_attr, FB_SMEM));
    attr = true;
  }
  const dim3 grid((unsigned)n, (unsigned)Hkv);
  if (a.diag)
    attn_bwd_tc_kernel<true><<<grid, FB_THREADS, FB_SMEM, stream>>>(mq, mk, mv, mdo, mdq, mdk, mdv, a);
  else
    attn_bwd_tc_kernel<false><<<grid, FB_THREADS, FB_SMEM, stream>>>(mq, mk, mv, mdo, mdq, mdk, mdv, a);
  ART_CUDA_CHECK(cudaGetLastError());
  return {dq, dk, dv, delta};
}

}  // namespace art
