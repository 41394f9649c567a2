// Host/device interface of the tcgen05 GEMM.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace atlas {

enum GemmEpilogue : int {
  kEpiStore = 0,     // out[n, m] = acc           (activation dtype)
  kEpiResidual = 1,  // out[n, m] += acc          (fp32 residual stream)
  kEpiSilu = 2,      // out[n, f] = silu(gate) * up for 64+64 interleaved rows
  kEpiF32 = 3,       // out[n, m] = acc           (fp32, e.g. logits)
  kEpiPeer = 4,      // dst_r[n, m] = acc for every destination r (fp32, peer GPUs), then signal
};

constexpr int kMaxPeers = 8;

// Destinations of the peer epilogue: the fp32 tile goes to `ndst` buffers
// (this GPU's or other GPUs' memory, mapped by CUDA IPC), all with row stride
// `ldo`.  When every CTA of the launch has stored its tile, the last one bumps
// the local sequence number `seq` and release-stores it into each
// destination's flag word for this rank.
struct PeerOut {
  int ndst;
  float* dst[kMaxPeers];
  uint32_t* flag[kMaxPeers];
  uint32_t* ticket;  // local, zero between launches
  uint32_t* seq;     // local
};

struct GemmParams {
  int M;             // output features (rows of A)
  int N;             // tokens (rows of B)
  int K;             // reduction length
  int ldo;           // leading dimension of `out` (elements)
  int splits;        // split-K factor = cluster size along z (1..8)
  int kb_per_split;  // 64-wide K blocks per split
  int bf16;          // operands are bf16 (else fp16)
  void* out;
  int* err;          // device error flag
  PeerOut peer;      // kEpiPeer only
};

void launch_gemm_tn(const CUtensorMap& a, const CUtensorMap& b, const GemmParams& p, int bn, int epi,
                    cudaStream_t st);
int gemm_smem_bytes(int bn);

}  // namespace atlas
