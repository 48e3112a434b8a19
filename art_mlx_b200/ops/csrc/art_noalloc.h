// Allocation-free C entry point of the prefix-tree attention backward.
//
// This declaration has no counterpart in the reference, which has no native
// code.  It serves callers that cannot allocate device memory themselves: a
// host application that owns the whole device memory budget and hands a
// plugin fixed buffers, or a latency-critical loop that must never enter the
// CUDA allocator (cudaMalloc/cudaFree can synchronise the device).  Such a
// caller passes every input and output; the only scratch the backward needs,
// the per-(head, query) vector delta = sum_d(dO * O), lives in a file-scope
// device array of the library (ART_NOALLOC_DELTA_MAX floats = 4 MiB), which
// every GPU that loads the library holds until the process exits.
//
// Layouts (all pointers are device addresses on the current device):
//   dout, q, out : bf16 rows of T x Hq x 128, row strides lddo / ldq / ldo (elements)
//   k, v         : bf16 rows of T x Hkv x 128, row strides ldk / ldv (elements)
//   lse          : fp32 [Hq, T] natural-log logsumexp of the forward
//   kend         : int32 [T], key j is visible to query i iff j <= i < kend[j]
//   units        : int32 [n_units, 3] contiguous, rows (key block of 128,
//                  first query tile, end query tile) in 32-query tiles;
//                  entries outside the sequence are skipped by the kernel
//   dq           : fp32 [T, Hq, 128] contiguous; dk, dv: fp32 [T, Hkv, 128] contiguous
// The outputs are cleared by the entry point before accumulation.
//
// Every row stride must be a multiple of 8 elements, at least H * 128 for its
// operand, and every bf16 base address 16-byte aligned; the fp32 outputs must
// be 16-byte aligned.
//
// Behaviour:
//  * the device address of the scratch array is looked up on every call
//    (cudaGetSymbolAddress, which allocates nothing), with the caller's device
//    current, so nothing goes stale after a device reset;
//  * all calls on one device share the scratch array and it keeps the last
//    call's contents; calls that overlap on the GPU (different streams with no
//    ordering between them) race on it: order them on one stream;
//  * no cudaMalloc, cudaFree or allocating library routine is called.
#ifndef ART_NOALLOC_H_
#define ART_NOALLOC_H_

#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

// Return codes.
enum {
  ART_NOALLOC_OK = 0,
  ART_NOALLOC_CUDA_ERROR = 1,       // a CUDA call or kernel launch of this entry point failed
  ART_NOALLOC_TOO_LARGE = 2,        // T * Hq > ART_NOALLOC_DELTA_MAX
  ART_NOALLOC_BAD_HEAD_DIM = 3,     // head_dim other than 128
  ART_NOALLOC_BAD_ARGUMENT = 4,     // sizes, null pointers, strides or alignment
};

#define ART_NOALLOC_DELTA_MAX (((int64_t)1) << 20)  // floats of scratch per device

int art_attn_bwd_noalloc(const void* dout, int64_t lddo, const void* q, int64_t ldq, const void* k, int64_t ldk,
                         const void* v, int64_t ldv, const void* out, int64_t ldo, const float* lse, const int* kend,
                         const int* units, int n_units, float* dq, float* dk, float* dv, int T, int Hq, int Hkv,
                         int D, float scale, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif  // ART_NOALLOC_H_
