// Allocation-free entry point for the vocabulary log-softmax + top-k.
//
// This entry point has no counterpart in the reference implementation; it is
// an addition of this library.
//
// Who needs it: callers that must not allocate device memory while they
// serve -- a host process whose device-memory budget is fixed and accounted
// when it starts (so a late cudaMalloc may fail under pressure or fragment the
// arena), a foreign runtime that owns the device allocator and does not want
// allocations made behind its back, or plain C/C++ code that links this
// library without PyTorch's caching allocator.  The regular binding (`topk`)
// allocates its per-call scratch through PyTorch; this one allocates nothing.
//
// How: the per-(row, chunk) partial records live in one file-scope device
// array of 4096 records x 26 floats (416 KiB).  Every GPU that loads the
// library holds that array until the process exits.  The caller still owns
// and passes the logits and the two output arrays.
//
// Contract:
//  * The first call on a device resolves the array's device address
//    (cudaGetSymbolAddress with that device current).  Make that first call
//    before any stream capture on the device.
//  * All calls on a device share the one array, which keeps the previous
//    call's contents.  Nothing in it has to start at zero: each call writes
//    every record it later reads.  Calls that overlap on the GPU (different
//    streams without ordering between them) race on the array and give wrong
//    results -- order them.
//  * rows x chunks must fit in 4096 records, where chunks is the vocabulary
//    split the kernel uses (see the .cu file); larger requests are rejected
//    with ATLAS_NOALLOC_ETOOLARGE and a message on stderr, before any launch.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define ATLAS_NOALLOC_OK 0
#define ATLAS_NOALLOC_EINVAL (-1)    // bad argument (null pointer, rows/vocab < 1, k outside 1..8)
#define ATLAS_NOALLOC_ETOOLARGE (-2) // rows x chunks exceeds the fixed scratch
#define ATLAS_NOALLOC_ECUDA (-3)     // CUDA error while resolving the scratch address or launching

#ifdef __cplusplus
extern "C" {
#endif

// logits [rows, vocab] fp32 (device) -> out_logprobs [rows, k] fp32 and
// out_ids [rows, k] int64 (device): per row, the k largest entries (greedy,
// keys == NULL) or a keyed Gumbel-top-k sample (keys: one int64 per row,
// scores logit * inv_temperature + noise), with untempered log-probabilities.
// Enqueued on `stream`; returns one of the ATLAS_NOALLOC_* codes.
__attribute__((visibility("default"))) int atlas_topk_logprobs_noalloc(
    const float* logits, int rows, int vocab, int k, const int64_t* keys, float inv_temperature,
    float* out_logprobs, int64_t* out_ids, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
