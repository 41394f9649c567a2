// Host/device interface of the block-scaled fp8 GEMM and its quantizers.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gemm.h"

namespace atlas {

constexpr int kFp8MaxKbPerCta = 64;  // 128-wide K blocks one CTA covers (scales staged in shared memory)

struct Fp8GemmParams {
  int M;             // output features (rows of Wq)
  int N;             // tokens (rows of Xq)
  int K;             // reduction length (multiple of 128)
  int ldo;           // leading dimension of `out` (elements)
  int splits;        // split-K factor = cluster size along z (1..8)
  int kb_per_split;  // 128-wide K blocks per split (<= kFp8MaxKbPerCta)
  int out_bf16;      // activation-dtype outputs are bf16 (else fp16)
  int lds;           // row stride of `sa` (>= N)
  const float* sw;   // weight scales [ceil(M/128)][K/128]
  const float* sa;   // activation scales [K/128][lds]
  void* out;
  int* err;
  PeerOut peer;      // kEpiPeer only
  int stream_hint;   // load weight tiles with the evict-first L2 policy (read once per forward)
};

void launch_gemm_fp8(const CUtensorMap& a, const CUtensorMap& b, const Fp8GemmParams& p, int bn, int epi,
                     cudaStream_t st);
int gemm_fp8_smem_bytes(int bn);
void launch_quant_fp8(const void* x, uint8_t* xq, float* sa, int N, int K, int lds, bool bf16, cudaStream_t st);
void launch_rmsnorm_fp8(const float* h, const void* w, uint8_t* xq, float* sa, int N, int H, int lds, float eps,
                        bool bf16, cudaStream_t st);

}  // namespace atlas
