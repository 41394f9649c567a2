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
  kEpiResidualNorm = 5,  // residual add, plus the activation-dtype copy of h and per-tile sums of h^2
  kEpiRope = 6,      // QKV: rotary embedding on q/k heads, q to q_out, k/v appended to the paged KV cache
};

// RMSNorm folded into a GEMM: the B operand is h in the activation dtype and
// the norm gain is folded into the weight rows, so the epilogue scales column
// n by rstd(n) = rsqrt(sum_t ss[t * ld + n] / H + eps), the sum running over
// the `tiles` per-128-feature partial sums (in tile order: deterministic).
struct NormIn {
  const float* ss;  // nullptr: no scaling
  int tiles;
  int ld;
  float inv_h;
  float eps;
};

// Extra outputs of kEpiResidualNorm: hb[n, m] = h (activation dtype) and
// ss[m / 128 * ld + n] = sum over the tile's 128 features of h^2.
struct NormOut {
  float* ss;
  int ld;
  void* hb;
};

// kEpiRope: tile m0 is one head of 128 dims (q heads, then k, then v).
struct RopeOut {
  const float* table;  // [max_pos, 128]: cos in [0, 64), sin in [64, 128)
  const int* pos;      // [N]
  const int* slots;    // [N] KV slot (page * ps + offset)
  void* kv;            // layer [num_pages, 2, Hkv, ps, 128]
  void* q;             // [N, Hq, 128]
  int Hq, Hkv, ps, num_pages, max_pos;
};

constexpr int kMaxPeers = 8;
// Bit pattern marking an unwritten receive slot: a NaN that IEEE arithmetic
// on the GPU never produces (its canonical NaN is 0x7fffffff); a computed
// value with this pattern is stored as the canonical NaN instead.
constexpr uint32_t kPeerSentinel = 0xffffffffu;

// Destinations of the peer epilogue: the fp32 tile goes to `ndst` buffers
// (this GPU's or other GPUs' memory, mapped by CUDA IPC), all with row stride
// `ldo`.  When every CTA of the launch has stored its tile, the last one bumps
// the local sequence number `seq` and release-stores it into each
// destination's flag word for this rank.
struct PeerOut {
  int ndst;
  int sentinel;      // 1: receive buffers hold kPeerSentinel until written; no fence, ticket or flags
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
  NormIn nin;        // optional rstd column scaling (store, SiLU, fp32, rope epilogues)
  NormOut nout;      // kEpiResidualNorm only
  RopeOut rope;      // kEpiRope only
  int stream_hint;   // load weight tiles with the evict-first L2 policy (read once per forward)
};

void launch_gemm_tn(const CUtensorMap& a, const CUtensorMap& b, const GemmParams& p, int bn, int epi,
                    cudaStream_t st);
int gemm_smem_bytes(int bn);

}  // namespace atlas
