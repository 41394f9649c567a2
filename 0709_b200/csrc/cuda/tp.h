// Launch wrappers of the tensor-parallel reduction kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace atlas {

// h[M, H] += sum over nsrc slots of recv[slot * slot_stride + m * H + i] (rank
// order), after waiting for flags[0..nsrc) >= *seq when flags != nullptr;
// then x = rmsnorm(h) * gamma unless gamma == nullptr.
// sentinel != 0: no flags; each float4 of a slot is polled until it holds no
// sentinel word, then reset to the sentinel (see PeerOut::sentinel).
void launch_tp_reduce_rmsnorm(const float* recv, int64_t slot_stride, const uint32_t* flags, const uint32_t* seq,
                              int nsrc, int sentinel, float* h, const void* gamma, void* x, int M, int H, float eps,
                              bool bf16, int* err, cudaStream_t st);
void launch_tp_wait(const uint32_t* flags, const uint32_t* seq, int nsrc, int* err, cudaStream_t st);

// Wall-time limit (ns) of the cross-GPU waits of the kernels above, on the current device.
cudaError_t set_peer_wait_ns(uint64_t ns);
cudaError_t get_peer_wait_ns(uint64_t* ns);

}  // namespace atlas
