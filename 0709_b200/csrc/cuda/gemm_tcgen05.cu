// tcgen05 GEMM for sm_100a:  D[m, n] = sum_k A[m, k] * B[n, k]
//
// A is the weight matrix [M_out, K] (K-major) and B the activations
// [N_tok, K] (K-major): "swap-AB", so the 128-row MMA dimension runs over
// output features and the small token count is the MMA N dimension (16..256).
// The same kernel serves decode/verify (N_tok <= 64, weight-bandwidth bound,
// split-K to fill all SMs) and prefill (N_tok up to 8192, 256-token tiles).
//
// Pipeline per CTA (128 threads):
//   thread 0   TMA producer: 128x64 weight tile + BNx64 activation tile per
//              stage into a STAGES-deep ring of 128B-swizzled shared memory;
//   thread 32  MMA issuer: 4 x tcgen05.mma (M=128, N=BN, K=16) per stage into
//              a TMEM accumulator, tcgen05.commit releases the stage;
//   all        epilogue: tcgen05.ld the 128 x BN fp32 accumulator (lane =
//              output feature) and apply the fused epilogue.
// Split-K partials go to a fp32 workspace; the last CTA of a tile (atomic
// ticket) sums the partials in split order, so results are deterministic
// and independent of the batch composition.

#include <cuda.h>

#include "common.cuh"
#include "gemm.h"
#include "launch.h"

namespace atlas {

template <int BN>
struct GemmSmem {
  static constexpr int kABytes = 128 * 128;  // 128 rows x 64 K x 2 B
  static constexpr int kBBytes = BN * 128;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = (BN <= 16) ? 6 : (BN <= 32 ? 5 : (BN <= 64 ? 4 : (BN <= 128 ? 4 : 3)));
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
  static constexpr int kBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
};

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }

template <int BN, int EPI, typename T>
__device__ __forceinline__ void epilogue_chunk(const GemmParams& p, int m0, int n0, int c0, const float* v,
                                               float* xchg) {
  const int tid = threadIdx.x;
  if constexpr (EPI == kEpiSilu) {
    // Rows 0..63 of the tile are gate features, 64..127 the matching up features.
    float* ex = xchg;  // [32 cols][64]
    if (tid >= 64) {
#pragma unroll
      for (int j = 0; j < 32; ++j) ex[j * 64 + (tid - 64)] = v[j];
    }
    __syncthreads();
    if (tid < 64) {
      const int f = (m0 >> 1) + tid;
      T* out = reinterpret_cast<T*>(p.out);
#pragma unroll 4
      for (int j = 0; j < 32; ++j) {
        const int n = n0 + c0 + j;
        if (n < p.N && f < (p.M >> 1)) out[static_cast<int64_t>(n) * p.ldo + f] = from_f32<T>(silu_f(v[j]) * ex[j * 64 + tid]);
      }
    }
    __syncthreads();
  } else {
    const int m = m0 + tid;
    if (m >= p.M) return;
#pragma unroll 4
    for (int j = 0; j < 32; ++j) {
      const int n = n0 + c0 + j;
      if (n >= p.N) break;
      const int64_t idx = static_cast<int64_t>(n) * p.ldo + m;
      if constexpr (EPI == kEpiStore) {
        reinterpret_cast<T*>(p.out)[idx] = from_f32<T>(v[j]);
      } else if constexpr (EPI == kEpiResidual) {
        float* r = reinterpret_cast<float*>(p.out);
        r[idx] = r[idx] + v[j];
      } else {  // kEpiF32
        reinterpret_cast<float*>(p.out)[idx] = v[j];
      }
    }
  }
}

template <int BN, int EPI, typename T>
__global__ void __launch_bounds__(128, 1)
    gemm_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmParams p) {
  using S = GemmSmem<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kStages * S::kStageBytes);
  uint64_t* empty = full + S::kStages;
  uint64_t* done = empty + S::kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  int* flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int m0 = blockIdx.x * 128;
  const int n0 = blockIdx.y * BN;
  const int split = blockIdx.z;
  const int kb_total = (p.K + 63) / 64;
  const int kb0 = split * p.kb_per_split;
  const int kb1 = min(kb0 + p.kb_per_split, kb_total);
  const int nk = kb1 - kb0;

  if (tid == 0) {
    for (int s = 0; s < S::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 0) tmem_alloc(tmem_slot, S::kTmemCols);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();
  bool ok = true;

  if (tid == 0) {
    // Weight tiles do not depend on the previous kernel: stream the first
    // stages before waiting for it, then the activations.
    const int pre = min(nk, S::kStages);
    for (int i = 0; i < pre; ++i) {
      mbar_arrive_expect_tx(&full[i], S::kStageBytes);
      tma_load_2d(smem + i * S::kStageBytes, &tmA, &full[i], (kb0 + i) * 64, m0);
    }
    pdl_wait();
    for (int i = 0; i < pre; ++i)
      tma_load_2d(smem + i * S::kStageBytes + S::kABytes, &tmB, &full[i], (kb0 + i) * 64, n0);
    for (int i = pre; i < nk && ok; ++i) {
      const int s = i % S::kStages;
      ok = mbar_wait(&empty[s], ((i / S::kStages) - 1) & 1, p.err);
      if (!ok) break;
      uint8_t* a = smem + s * S::kStageBytes;
      uint8_t* b = a + S::kABytes;
      mbar_arrive_expect_tx(&full[s], S::kStageBytes);
      tma_load_2d(a, &tmA, &full[s], (kb0 + i) * 64, m0);
      tma_load_2d(b, &tmB, &full[s], (kb0 + i) * 64, n0);
    }
  } else if (tid == 32) {
    constexpr uint32_t idesc_h = umma_idesc_f16(128, BN, false, false, false);
    constexpr uint32_t idesc_b = umma_idesc_f16(128, BN, true, false, false);
    const uint32_t idesc = p.bf16 ? idesc_b : idesc_h;
    for (int i = 0; i < nk && ok; ++i) {
      const int s = i % S::kStages;
      ok = mbar_wait(&full[s], (i / S::kStages) & 1, p.err);
      if (!ok) break;
      tc_fence_after();
      const uint32_t a = smem_u32(smem + s * S::kStageBytes);
      const uint32_t b = a + S::kABytes;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        umma_f16_ss(tmem, umma_desc_sw128(a + kk * 32, 16, 1024), umma_desc_sw128(b + kk * 32, 16, 1024), idesc,
                    (i | kk) != 0 ? 1u : 0u);
      }
      umma_commit(&empty[s]);
    }
    umma_commit(done);
  }
  __syncwarp();
  pdl_wait();
  if (nk > 0) ok = mbar_wait(done, 0, p.err) && ok;
  tc_fence_after();
  if (tid == 0) *flag = ok ? 1 : 0;
  __syncthreads();
  ok = *flag != 0;

  float* xchg = reinterpret_cast<float*>(smem);  // stage buffers are free once `done` fired
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
  if (p.splits == 1) {
    for (int c0 = 0; c0 < BN; c0 += 32) {
      if (n0 + c0 >= p.N) break;
      float v[32];
      if (ok && nk > 0) {
        tmem_ld32(tmem + lane_base + c0, v);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.f;
      }
      epilogue_chunk<BN, EPI, T>(p, m0, n0, c0, v, xchg);
    }
  } else {
    // Write this split's partial tile: ws[split][n][m] (fp32).
    const int m = m0 + tid;
    for (int c0 = 0; c0 < BN; c0 += 32) {
      if (n0 + c0 >= p.N) break;
      float v[32];
      if (ok && nk > 0) {
        tmem_ld32(tmem + lane_base + c0, v);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.f;
      }
      if (m < p.M) {
        for (int j = 0; j < 32; ++j) {
          const int n = n0 + c0 + j;
          if (n >= p.N) break;
          p.ws[(static_cast<int64_t>(split) * p.N + n) * p.M + m] = v[j];
        }
      }
    }
    __threadfence();
    __syncthreads();
    const int tile = blockIdx.y * gridDim.x + blockIdx.x;
    if (tid == 0) *flag = (atomicAdd(&p.counters[tile], 1) == p.splits - 1) ? 1 : 0;
    __syncthreads();
    if (*flag) {
      __threadfence();
      for (int c0 = 0; c0 < BN; c0 += 32) {
        if (n0 + c0 >= p.N) break;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.f;
        if (m < p.M) {
          for (int s = 0; s < p.splits; ++s) {
            const float* src = p.ws + (static_cast<int64_t>(s) * p.N) * p.M + m;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int n = n0 + c0 + j;
              if (n < p.N) v[j] += __ldcg(src + static_cast<int64_t>(n) * p.M);
            }
          }
        }
        epilogue_chunk<BN, EPI, T>(p, m0, n0, c0, v, xchg);
      }
      if (tid == 0) p.counters[tile] = 0;  // ready for the next launch
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, S::kTmemCols);
}

// ------------------------------------------------------------------ host
template <int BN, int EPI, typename T>
static void launch_bn(const CUtensorMap& a, const CUtensorMap& b, const GemmParams& p, dim3 grid, cudaStream_t st) {
  using S = GemmSmem<BN>;
  auto kern = gemm_tn_kernel<BN, EPI, T>;
  static bool configured = false;  // per instantiation
  if (!configured) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kBytes);
    configured = true;
  }
  launch_k(kern, grid, dim3(128), S::kBytes, st, a, b, p);
}

template <int EPI, typename T>
static void launch_epi(int bn, const CUtensorMap& a, const CUtensorMap& b, const GemmParams& p, dim3 grid,
                       cudaStream_t st) {
  switch (bn) {
    case 16: launch_bn<16, EPI, T>(a, b, p, grid, st); break;
    case 32: launch_bn<32, EPI, T>(a, b, p, grid, st); break;
    case 64: launch_bn<64, EPI, T>(a, b, p, grid, st); break;
    case 128: launch_bn<128, EPI, T>(a, b, p, grid, st); break;
    default: launch_bn<256, EPI, T>(a, b, p, grid, st); break;
  }
}

void launch_gemm_tn(const CUtensorMap& a, const CUtensorMap& b, const GemmParams& p, int bn, int epi,
                    cudaStream_t st) {
  dim3 grid((p.M + 127) / 128, (p.N + bn - 1) / bn, p.splits);
  if (p.bf16) {
    switch (epi) {
      case kEpiStore: launch_epi<kEpiStore, __nv_bfloat16>(bn, a, b, p, grid, st); break;
      case kEpiResidual: launch_epi<kEpiResidual, __nv_bfloat16>(bn, a, b, p, grid, st); break;
      case kEpiSilu: launch_epi<kEpiSilu, __nv_bfloat16>(bn, a, b, p, grid, st); break;
      default: launch_epi<kEpiF32, __nv_bfloat16>(bn, a, b, p, grid, st); break;
    }
  } else {
    switch (epi) {
      case kEpiStore: launch_epi<kEpiStore, __half>(bn, a, b, p, grid, st); break;
      case kEpiResidual: launch_epi<kEpiResidual, __half>(bn, a, b, p, grid, st); break;
      case kEpiSilu: launch_epi<kEpiSilu, __half>(bn, a, b, p, grid, st); break;
      default: launch_epi<kEpiF32, __half>(bn, a, b, p, grid, st); break;
    }
  }
}

int gemm_smem_bytes(int bn) {
  switch (bn) {
    case 16: return GemmSmem<16>::kBytes;
    case 32: return GemmSmem<32>::kBytes;
    case 64: return GemmSmem<64>::kBytes;
    case 128: return GemmSmem<128>::kBytes;
    default: return GemmSmem<256>::kBytes;
  }
}

}  // namespace atlas
