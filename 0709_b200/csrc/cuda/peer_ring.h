// Launch wrappers of the peer message rings (see peer_ring.cu for the layout and protocol).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace atlas {

constexpr int kRingSlotOffset = 256;  // the message slot's offset in a ring allocation

// Copy `bytes` (header + payload, 16-byte aligned source) into the peer ring's
// slot and publish `seq` on its flag.
cudaError_t launch_ring_push(const void* src, int64_t bytes, void* peer_ring, uint32_t seq, cudaStream_t st);

// Wait (at most limit_ns) until the local ring's flag reaches `seq`, then copy
// header + payload to dst (at most dst_bytes); *out_nbytes = payload bytes, or
// -1 if nothing was copied (timeout: err = kErrPeerTimeout; too long or a
// stale header: err = kErrBadIndex).
cudaError_t launch_ring_pop(const void* ring, uint32_t seq, void* dst, int64_t dst_bytes, int* out_nbytes, int* err,
                            uint64_t limit_ns, cudaStream_t st);

}  // namespace atlas
