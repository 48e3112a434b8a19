// Peer-memory communication layer and the fused data-parallel LoRA update.
//
// * ipc_alloc / ipc_open / ipc_close: one cudaMalloc arena per rank exported
//   with CUDA IPC; every rank maps every peer's arena (NVLink P2P through
//   NVSwitch).  Kernels address peers through per-buffer base-pointer tables.
// * peer_barrier: cross-GPU barrier on flags in the arenas.  Each wait polls
//   with an iteration AND %globaltimer limit; on timeout it records an error
//   code in a local status word and returns (the host checks the status).
// * dp_reduce_sumsq + dp_adamw_allgather: the data-parallel optimizer step.
//   Rank r owns shard r of the flat LoRA buffers.  Phase 1 sums shard r of
//   every rank's fp32 gradient with P2P loads and takes its sum of squares;
//   after a barrier, phase 2 reads the peers' partial norms, clips, runs AdamW
//   on the shard (master weights and moments exist only for the shard) and
//   writes the bf16 parameters into every rank's compute buffer with P2P
//   stores; a final barrier publishes them.  No TMA / multicast loads touch
//   peer memory: all remote traffic is plain ld/st.global.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "common.cuh"

namespace art {

// ---------------------------------------------------------------- IPC arena
std::vector<torch::Tensor> ipc_alloc(int64_t nbytes) {
  void* ptr = nullptr;
  ART_CUDA_CHECK(cudaMalloc(&ptr, nbytes));
  ART_CUDA_CHECK(cudaMemset(ptr, 0, nbytes));
  cudaIpcMemHandle_t h;
  ART_CUDA_CHECK(cudaIpcGetMemHandle(&h, ptr));
  int dev = 0;
  ART_CUDA_CHECK(cudaGetDevice(&dev));
  auto opts = torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, dev);
  auto buf = torch::from_blob(ptr, {nbytes}, [](void* p) { cudaFree(p); }, opts);
  auto handle = torch::empty({(int64_t)sizeof(h)}, torch::kUInt8);
  memcpy(handle.data_ptr(), &h, sizeof(h));
  return {buf, handle};
}

int64_t ipc_open(torch::Tensor handle) {
  TORCH_CHECK(handle.numel() == (int64_t)sizeof(cudaIpcMemHandle_t) && handle.device().is_cpu());
  cudaIpcMemHandle_t h;
  memcpy(&h, handle.data_ptr(), sizeof(h));
  void* ptr = nullptr;
  ART_CUDA_CHECK(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(ptr);
}

void ipc_close(int64_t ptr) { ART_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr))); }

// ---------------------------------------------------------------- barrier
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// flags layout per rank arena: uint32 flags[world] (slot k written by rank k)
// status: local int32 error word (0 ok, 1 barrier timeout)
__global__ void peer_barrier_kernel(const int64_t* __restrict__ flag_bases, int rank, int world,
                                    uint32_t epoch, int64_t timeout_ns, int* __restrict__ status) {
  if (threadIdx.x == 0) {
    __threadfence_system();
  }
  __syncthreads();
  if (threadIdx.x < world) {
    uint32_t* peer_flags = reinterpret_cast<uint32_t*>(flag_bases[threadIdx.x]);
    st_release_sys(peer_flags + rank, epoch);
  }
  __syncthreads();
  if (threadIdx.x < world) {
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(flag_bases[rank]);
    const uint64_t t0 = globaltimer();
    // bounded spin: both an iteration cap and a wall-clock cap
    for (int64_t it = 0; it < (int64_t)1 << 31; ++it) {
      if ((int32_t)(ld_acquire_sys(mine + threadIdx.x) - epoch) >= 0) break;
      if ((int64_t)(globaltimer() - t0) > timeout_ns) {
        atomicExch(status, 1);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
}

void peer_barrier(torch::Tensor flag_bases, int64_t rank, int64_t world, int64_t epoch,
                  int64_t timeout_ns, torch::Tensor status) {
  TORCH_CHECK(world <= 32);
  peer_barrier_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      flag_bases.data_ptr<int64_t>(), (int)rank, (int)world, (uint32_t)epoch, timeout_ns,
      status.data_ptr<int>());
  ART_CUDA_CHECK(cudaGetLastError());
}

// ---------------------------------------------------------------- DP update
// Phase 1: g[shard] = sum_k grad_k[shard] (written into this rank's grad
// buffer), partial = sum g^2 (local scalar).
__global__ void dp_reduce_sumsq_kernel(const int64_t* __restrict__ grad_bases, int world,
                                       int64_t off, int64_t n, float* __restrict__ partial) {
  __shared__ float red[32];
  float acc = 0.f;
  const int rank_self = -1;
  (void)rank_self;
  float* mine = nullptr;
  // grad_bases[world] holds this rank's own (local) pointer
  mine = reinterpret_cast<float*>(grad_bases[world]) + off;
  const int64_t n4 = n / 4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < world; ++k) {
      const float4 v = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(grad_bases[k]) + off)[i];
      s.x += v.x;
      s.y += v.y;
      s.z += v.z;
      s.w += v.w;
    }
    reinterpret_cast<float4*>(mine)[i] = s;
    acc += s.x * s.x + s.y * s.y + s.z * s.z + s.w * s.w;
  }
  for (int64_t i = n4 * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < world; ++k) s += (reinterpret_cast<const float*>(grad_bases[k]) + off)[i];
    mine[i] = s;
    acc += s * s;
  }
  acc = block_sum(acc, red);
  if (threadIdx.x == 0) atomicAdd(partial, acc);
}

// Publish this rank's partial norm into slot `rank` of every peer's norm table.
__global__ void dp_publish_norm_kernel(const int64_t* __restrict__ norm_bases, int rank, int world,
                                       const float* __restrict__ partial) {
  if (threadIdx.x < world) {
    float* dst = reinterpret_cast<float*>(norm_bases[threadIdx.x]);
    dst[rank] = *partial;
  }
}

// Phase 2: clip, AdamW on the shard, bf16 all-gather by peer stores, zero grads.
// hp as in adamw_kernel.
__global__ void dp_adamw_allgather_kernel(const int64_t* __restrict__ compute_bases, int world,
                                          int64_t off, int64_t n, float* __restrict__ grad_shard,
                                          float* __restrict__ master, float* __restrict__ m,
                                          float* __restrict__ v, const float* __restrict__ hp,
                                          const float* __restrict__ norms,
                                          float* __restrict__ norm_out) {
  const float lr = hp[0], b1 = hp[1], b2 = hp[2], eps = hp[3], wd = hp[4], clip = hp[5];
  const float gs = hp[6], step = hp[7];
  float sq = 0.f;
  for (int k = 0; k < world; ++k) sq += norms[k];
  const float gnorm = sqrtf(sq) * gs;
  float coef = gs;
  if (clip > 0.f && gnorm > clip) coef *= clip / (gnorm + 1e-6f);
  if (norm_out && blockIdx.x == 0 && threadIdx.x == 0) *norm_out = gnorm;
  const float bc1 = 1.f - powf(b1, step), bc2 = 1.f - powf(b2, step);
  const float step_size = lr / bc1;
  const float inv_bc2_sqrt = rsqrtf(bc2);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float gi = grad_shard[i] * coef;
    const float mi = b1 * m[i] + (1.f - b1) * gi;
    const float vi = b2 * v[i] + (1.f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    float pi = master[i] * (1.f - lr * wd);
    pi -= step_size * mi / (sqrtf(vi) * inv_bc2_sqrt + eps);
    master[i] = pi;
    const __nv_bfloat16 b = f2bf(pi);
    for (int k = 0; k < world; ++k) reinterpret_cast<__nv_bfloat16*>(compute_bases[k])[off + i] = b;
  }
}

static int dp_grid(int64_t n) {
  int64_t b = (n + 255) / 256;
  if (b > 148 * 4) b = 148 * 4;
  return (int)(b < 1 ? 1 : b);
}

// grad_bases: int64 [world + 1] (peers' grad buffer bases, then the local one)
void dp_reduce_sumsq(torch::Tensor grad_bases, int64_t world, int64_t off, int64_t n,
                     torch::Tensor partial) {
  auto stream = at::cuda::getCurrentCUDAStream();
  partial.zero_();
  dp_reduce_sumsq_kernel<<<dp_grid(n / 4 + 1), 256, 0, stream>>>(
      grad_bases.data_ptr<int64_t>(), (int)world, off, n, partial.data_ptr<float>());
  ART_CUDA_CHECK(cudaGetLastError());
}

void dp_publish_norm(torch::Tensor norm_bases, int64_t rank, int64_t world, torch::Tensor partial) {
  dp_publish_norm_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      norm_bases.data_ptr<int64_t>(), (int)rank, (int)world, partial.data_ptr<float>());
  ART_CUDA_CHECK(cudaGetLastError());
}

void dp_adamw_allgather(torch::Tensor compute_bases, int64_t world, int64_t off, int64_t n,
                        torch::Tensor grad_shard, torch::Tensor master, torch::Tensor m,
                        torch::Tensor v, torch::Tensor hp, torch::Tensor norms,
                        torch::Tensor norm_out) {
  TORCH_CHECK(grad_shard.numel() == n && master.numel() == n && m.numel() == n && v.numel() == n);
  dp_adamw_allgather_kernel<<<dp_grid(n), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      compute_bases.data_ptr<int64_t>(), (int)world, off, n, grad_shard.data_ptr<float>(),
      master.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), hp.data_ptr<float>(),
      norms.data_ptr<float>(), norm_out.data_ptr<float>());
  ART_CUDA_CHECK(cudaGetLastError());
}

}  // namespace art

namespace art {

// Copy nbytes from a peer's mapped buffer (CUDA-IPC address, reached over
// NVLink) into a local tensor, on the current stream (one copy-engine
// transfer; the SMs stay free for the GEMM that overlaps it).
void peer_copy(torch::Tensor dst, int64_t src_ptr, int64_t nbytes) {
  TORCH_CHECK(dst.is_cuda() && dst.is_contiguous() && dst.numel() * dst.element_size() >= nbytes);
  ART_CUDA_CHECK(cudaMemcpyAsync(dst.data_ptr(), reinterpret_cast<const void*>(src_ptr), (size_t)nbytes,
                                 cudaMemcpyDeviceToDevice, at::cuda::getCurrentCUDAStream()));
}

}  // namespace art
