// Block-scaled fp8 GEMM for sm_100a:
//   D[m, n] = sum_kb  sw[m/128, kb] * sa[kb, n] * sum_{k in kb} Wq[m, k] * Xq[n, k]
// with e4m3 weights Wq [M, K] scaled per 128x128 block (sw) and e4m3
// activations Xq [N, K] scaled per token per 128 columns (sa, stored
// kb-major as [KB][lds]).
//
// Same swap-AB tiling as the bf16 kernel (128 weight rows on the MMA M side,
// BN = 16..64 tokens as N), with 128-element (128-byte) K blocks so every
// K block has one weight scale per CTA tile.  Each K block's product goes to
// its own TMEM accumulator (two, alternating), where
//   warp 4      TMA producer (weights stream before griddepcontrol.wait),
//   warp 5      MMA issuer: 4 x tcgen05.mma.kind::f8f6f4 (K = 32) per block,
//   warps 0..3  promotion: tcgen05.ld the block's 128 x BN fp32 product,
//               release the accumulator, and add it into registers scaled by
//               sw * sa[n]  (lane = output feature, register = token).
// Split-K CTAs form a cluster and reduce their register tiles through
// distributed shared memory, then the same epilogues as the bf16 kernel
// (store / residual / SiLU-mul / fp32 / peer stores) run.

#include <cuda.h>
#include <cuda_fp8.h>

#include "common.cuh"
#include "gemm.h"
#include "gemm_fp8.h"
#include "launch.h"

namespace atlas {

template <int BN>
struct Fp8Smem {
  static constexpr int kABytes = 128 * 128;  // 128 rows x 128 K x 1 B
  static constexpr int kBBytes = BN * 128;
  static constexpr int kStageBytes = kABytes + kBBytes;
  // BN <= 32: ~96 KB of shared memory and 256 TMEM columns, so two CTAs share an SM.
  static constexpr int kStages = BN <= 16 ? 5 : (BN <= 32 ? 4 : 6);
  static constexpr int kAccStride = BN < 32 ? 32 : BN;  // TMEM columns per accumulator
  // Accumulators in flight: the MMA warp runs up to kAccBufs K blocks ahead of
  // the promotion warps, so promotion latency does not throttle the stream.
  static constexpr int kAccBufs = 256 / kAccStride;     // 8 (BN <= 32) or 4 (BN = 64)
  static constexpr int kTmemCols = kAccBufs * kAccStride;  // 256
  static constexpr int kScaleBytes = kFp8MaxKbPerCta * (BN + 1) * 4;
  static constexpr int kPartBytes = BN * 128 * 4;       // split-K partial (reuses the stages)
  static constexpr int kBytes = kStages * kStageBytes + kScaleBytes + 1024 /*align*/ + 512 /*barriers*/;
  static_assert(kPartBytes <= kStages * kStageBytes, "partial tile must fit in the stage ring");
};

__device__ __forceinline__ float silu8(float x) { return x / (1.0f + __expf(-x)); }

__device__ __forceinline__ void umma_f8_ss(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Named barrier over the 128 promotion threads (warps 0..3).
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

template <int EPI, typename T>
__device__ __forceinline__ void fp8_store(const Fp8GemmParams& p, int m, int n, float v) {
  const int64_t idx = static_cast<int64_t>(n) * p.ldo + m;
  if constexpr (EPI == kEpiStore) {
    reinterpret_cast<T*>(p.out)[idx] = from_f32<T>(v);
  } else if constexpr (EPI == kEpiResidual) {
    float* r = reinterpret_cast<float*>(p.out);
    r[idx] = r[idx] + v;
  } else if constexpr (EPI == kEpiPeer) {
    const float w = (__float_as_uint(v) == kPeerSentinel) ? __uint_as_float(0x7fffffffu) : v;
    for (int r = 0; r < p.peer.ndst; ++r) p.peer.dst[r][idx] = w;
  } else {
    reinterpret_cast<float*>(p.out)[idx] = v;
  }
}

template <typename T>
__device__ __forceinline__ void fp8_store_silu(const Fp8GemmParams& p, int m0, int row, int n, float g, float u) {
  const int f = (m0 >> 1) + row;
  if (f < (p.M >> 1)) reinterpret_cast<T*>(p.out)[static_cast<int64_t>(n) * p.ldo + f] = from_f32<T>(silu8(g) * u);
}

template <int EPI>
__device__ __forceinline__ void fp8_peer_signal(const Fp8GemmParams& p) {
  if constexpr (EPI == kEpiPeer) {
    if (p.peer.sentinel) return;
    __syncthreads();
    if (threadIdx.x == 0) {
      fence_acq_rel_sys();
      const uint32_t total = gridDim.x * gridDim.y * gridDim.z;
      if (atomicAdd(p.peer.ticket, 1u) == total - 1) {
        *reinterpret_cast<volatile uint32_t*>(p.peer.ticket) = 0u;
        fence_acq_rel_sys();
        const uint32_t s = *reinterpret_cast<volatile uint32_t*>(p.peer.seq) + 1u;
        *reinterpret_cast<volatile uint32_t*>(p.peer.seq) = s;
        for (int r = 0; r < p.peer.ndst; ++r) st_release_sys(p.peer.flag[r], s);
      }
    }
  }
}

template <int BN, int EPI, typename T>
__global__ void __launch_bounds__(192, BN <= 32 ? 2 : 1)
    gemm_fp8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    Fp8GemmParams p) {
  using S = Fp8Smem<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* sa_s = reinterpret_cast<float*>(smem + S::kStages * S::kStageBytes);  // [nk][BN]
  float* sw_s = sa_s + kFp8MaxKbPerCta * BN;                                      // [nk]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kStages * S::kStageBytes + S::kScaleBytes);
  uint64_t* empty = full + S::kStages;
  uint64_t* tfull = empty + S::kStages;
  uint64_t* tempty = tfull + S::kAccBufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + S::kAccBufs);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int m0 = blockIdx.x * 128;
  const int n0 = blockIdx.y * BN;
  const int kb_total = p.K / 128;
  const int kb0 = blockIdx.z * p.kb_per_split;
  const int kb1 = min(kb0 + p.kb_per_split, kb_total);
  const int nk = max(0, kb1 - kb0);

  if (tid == 128) {
    for (int s = 0; s < S::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < S::kAccBufs; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);  // one arrival per promotion warp
    }
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 4) tmem_alloc(tmem_slot, S::kTmemCols);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();

  float acc[BN];
#pragma unroll
  for (int j = 0; j < BN; ++j) acc[j] = 0.f;

  if (warp == 4) {
    if (lane == 0) {
      bool ok = true;
      const bool hint = p.stream_hint != 0;
      const uint64_t pol = l2_policy_evict_first();
      const int pre = min(nk, S::kStages);
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], S::kStageBytes);
        if (hint)
          tma_load_2d_hint(smem + i * S::kStageBytes, &tmA, &full[i], (kb0 + i) * 128, m0, pol);
        else
          tma_load_2d(smem + i * S::kStageBytes, &tmA, &full[i], (kb0 + i) * 128, m0);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i)
        tma_load_2d(smem + i * S::kStageBytes + S::kABytes, &tmB, &full[i], (kb0 + i) * 128, n0);
      for (int i = pre; i < nk && ok; ++i) {
        const int s = i % S::kStages;
        ok = mbar_wait(&empty[s], ((i / S::kStages) - 1) & 1, p.err);
        if (!ok) break;
        uint8_t* a = smem + s * S::kStageBytes;
        mbar_arrive_expect_tx(&full[s], S::kStageBytes);
        if (hint)
          tma_load_2d_hint(a, &tmA, &full[s], (kb0 + i) * 128, m0, pol);
        else
          tma_load_2d(a, &tmA, &full[s], (kb0 + i) * 128, m0);
        tma_load_2d(a + S::kABytes, &tmB, &full[s], (kb0 + i) * 128, n0);
      }
    }
    __syncwarp();
  } else if (warp == 5) {
    if (lane == 0) {
      // kind::f8f6f4 with e4m3 A and B (format code 0) and fp32 accumulation.
      constexpr uint32_t idesc = umma_idesc_f16(128, BN, false, false, false);
      bool ok = true;
      for (int i = 0; i < nk && ok; ++i) {
        const int s = i % S::kStages;
        const int b = i % S::kAccBufs;
        const int u = i / S::kAccBufs;
        ok = mbar_wait(&full[s], (i / S::kStages) & 1, p.err);
        if (ok && u >= 1) ok = mbar_wait(&tempty[b], (u - 1) & 1, p.err);
        if (!ok) break;
        tc_fence_after();
        const uint32_t a = smem_u32(smem + s * S::kStageBytes);
        const uint32_t bb = a + S::kABytes;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_f8_ss(tmem + b * S::kAccStride, umma_desc_sw128(a + kk * 32, 16, 1024),
                     umma_desc_sw128(bb + kk * 32, 16, 1024), idesc, kk != 0 ? 1u : 0u);
        umma_commit(&empty[s]);
        umma_commit(&tfull[b]);
      }
    }
    __syncwarp();
  } else {
    // Promotion warps: stage this tile's scales, then fold each K block in.
    pdl_wait();
    const int mb = m0 / 128;
    for (int idx = tid; idx < nk * BN; idx += 128) {
      const int i = idx / BN, j = idx % BN;
      sa_s[idx] = (n0 + j < p.N) ? p.sa[static_cast<int64_t>(kb0 + i) * p.lds + n0 + j] : 0.f;
    }
    for (int i = tid; i < nk; i += 128) sw_s[i] = p.sw[static_cast<int64_t>(mb) * kb_total + kb0 + i];
    epi_bar();
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    for (int i = 0; i < nk; ++i) {
      const int b = i % S::kAccBufs;
      if (!mbar_wait(&tfull[b], (i / S::kAccBufs) & 1, p.err)) break;
      tc_fence_after();
      float v[BN < 32 ? 32 : BN];
#pragma unroll
      for (int c0 = 0; c0 < BN; c0 += 32) tmem_ld32(tmem + lane_base + b * S::kAccStride + c0, v + c0);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
      const float w = sw_s[i];
      const float* sa_row = sa_s + i * BN;
#pragma unroll
      for (int j = 0; j < BN; ++j) acc[j] = fmaf(v[j], w * sa_row[j], acc[j]);
    }
  }

  // ---------------------------------------------------------------- epilogue
  __syncthreads();
  const int ncols = min(BN, p.N - n0);
  if (p.splits == 1) {
    float* ex = reinterpret_cast<float*>(smem);  // [BN][64] gate/up exchange
    if constexpr (EPI == kEpiSilu) {
      if (tid >= 64 && tid < 128) {
#pragma unroll
        for (int j = 0; j < BN; ++j) ex[j * 64 + (tid - 64)] = acc[j];
      }
      __syncthreads();
      if (tid < 64) {
#pragma unroll
        for (int j = 0; j < BN; ++j)
          if (j < ncols) fp8_store_silu<T>(p, m0, tid, n0 + j, acc[j], ex[j * 64 + tid]);
      }
    } else {
      if (tid < 128 && m0 + tid < p.M) {
#pragma unroll
        for (int j = 0; j < BN; ++j)
          if (j < ncols) fp8_store<EPI, T>(p, m0 + tid, n0 + j, acc[j]);
      }
    }
  } else {
    float* part = reinterpret_cast<float*>(smem);  // [BN][128]
    if (tid < 128) {
#pragma unroll
      for (int j = 0; j < BN; ++j) part[j * 128 + tid] = acc[j];
    }
    const int NS = p.splits;
    cluster_sync();
    const uint32_t rank = cluster_ctarank();
    if (tid < 128) {
      for (int c = static_cast<int>(rank); c < ncols; c += NS) {
        const int n = n0 + c;
        if constexpr (EPI == kEpiSilu) {
          if (tid < 64) {
            float g = 0.f, u = 0.f;
            for (int s2 = 0; s2 < NS; ++s2) {
              g += ld_dsmem_f32(part + c * 128 + tid, s2);
              u += ld_dsmem_f32(part + c * 128 + 64 + tid, s2);
            }
            fp8_store_silu<T>(p, m0, tid, n, g, u);
          }
        } else if (m0 + tid < p.M) {
          float a = 0.f;
          for (int s2 = 0; s2 < NS; ++s2) a += ld_dsmem_f32(part + c * 128 + tid, s2);
          fp8_store<EPI, T>(p, m0 + tid, n, a);
        }
      }
    }
    cluster_sync();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 4) tmem_dealloc(tmem, S::kTmemCols);
  fp8_peer_signal<EPI>(p);
}

// ------------------------------------------------------------ quantization
// One warp per (row, 128-column block): amax, scale = amax / 448, e4m3 values.
__device__ __forceinline__ void quant_block_warp(const float (&v)[4], uint8_t* dst, float* scale_out, int lane) {
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
  amax = warp_max(amax);
  const float scale = fmaxf(amax, 1e-10f) * (1.0f / 448.0f);
  const float inv = 1.0f / scale;
  uint32_t packed = 0;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const __nv_fp8_storage_t q = __nv_cvt_float_to_fp8(v[e] * inv, __NV_SATFINITE, __NV_E4M3);
    packed |= static_cast<uint32_t>(q) << (8 * e);
  }
  *reinterpret_cast<uint32_t*>(dst + lane * 4) = packed;
  if (lane == 0) *scale_out = scale;
}

// x [N, K] (activation dtype) -> xq [N, K] e4m3, sa [K/128][lds]; grid (N), 256 threads.
template <typename T>
__global__ void quant_fp8_kernel(const T* __restrict__ x, uint8_t* __restrict__ xq, float* __restrict__ sa, int K,
                                 int lds) {
  pdl_wait();
  pdl_trigger();
  const int n = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const T* row = x + static_cast<int64_t>(n) * K;
  for (int kb = warp; kb < K / 128; kb += blockDim.x >> 5) {
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = to_f32(row[kb * 128 + lane * 4 + e]);
    quant_block_warp(v, xq + static_cast<int64_t>(n) * K + kb * 128, sa + static_cast<int64_t>(kb) * lds + n, lane);
  }
}

// RMSNorm of the fp32 residual row straight to e4m3 + scales; grid (N), 256 threads.
template <typename T>
__global__ void rmsnorm_fp8_kernel(const float* __restrict__ h, const T* __restrict__ w, uint8_t* __restrict__ xq,
                                   float* __restrict__ sa, int H, int lds, float eps) {
  pdl_wait();
  pdl_trigger();
  const int n = blockIdx.x;
  const float* row = h + static_cast<int64_t>(n) * H;
  float ss = 0.f;
  for (int i = threadIdx.x * 4; i < H; i += blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4*>(row + i);
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  __shared__ float red[32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) tot += red[i];
  const float inv = rsqrtf(tot / static_cast<float>(H) + eps);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int kb = warp; kb < H / 128; kb += blockDim.x >> 5) {
    const int c = kb * 128 + lane * 4;
    const float4 x4 = *reinterpret_cast<const float4*>(row + c);
    float v[4] = {x4.x * inv * to_f32(w[c]), x4.y * inv * to_f32(w[c + 1]), x4.z * inv * to_f32(w[c + 2]),
                  x4.w * inv * to_f32(w[c + 3])};
    quant_block_warp(v, xq + static_cast<int64_t>(n) * H + kb * 128, sa + static_cast<int64_t>(kb) * lds + n, lane);
  }
}

// ------------------------------------------------------------------- host
template <int BN, int EPI, typename T>
static void launch_fp8_bn(const CUtensorMap& a, const CUtensorMap& b, const Fp8GemmParams& p, dim3 grid,
                          cudaStream_t st) {
  using S = Fp8Smem<BN>;
  auto kern = gemm_fp8_kernel<BN, EPI, T>;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kBytes);
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = S::kBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = static_cast<unsigned>(p.splits);
  cfg.attrs = attr;
  cfg.numAttrs = p.splits > 1 ? 2 : 1;
  cudaLaunchKernelEx(&cfg, kern, a, b, p);
}

template <int EPI, typename T>
static void launch_fp8_epi(int bn, const CUtensorMap& a, const CUtensorMap& b, const Fp8GemmParams& p, dim3 grid,
                           cudaStream_t st) {
  switch (bn) {
    case 16: launch_fp8_bn<16, EPI, T>(a, b, p, grid, st); break;
    case 32: launch_fp8_bn<32, EPI, T>(a, b, p, grid, st); break;
    default: launch_fp8_bn<64, EPI, T>(a, b, p, grid, st); break;
  }
}

template <typename T>
static void launch_fp8_t(int bn, int epi, const CUtensorMap& a, const CUtensorMap& b, const Fp8GemmParams& p,
                         dim3 grid, cudaStream_t st) {
  switch (epi) {
    case kEpiStore: launch_fp8_epi<kEpiStore, T>(bn, a, b, p, grid, st); break;
    case kEpiResidual: launch_fp8_epi<kEpiResidual, T>(bn, a, b, p, grid, st); break;
    case kEpiSilu: launch_fp8_epi<kEpiSilu, T>(bn, a, b, p, grid, st); break;
    case kEpiPeer: launch_fp8_epi<kEpiPeer, T>(bn, a, b, p, grid, st); break;
    default: launch_fp8_epi<kEpiF32, T>(bn, a, b, p, grid, st); break;
  }
}

void launch_gemm_fp8(const CUtensorMap& a, const CUtensorMap& b, const Fp8GemmParams& p, int bn, int epi,
                     cudaStream_t st) {
  dim3 grid((p.M + 127) / 128, (p.N + bn - 1) / bn, p.splits);
  if (p.out_bf16)
    launch_fp8_t<__nv_bfloat16>(bn, epi, a, b, p, grid, st);
  else
    launch_fp8_t<__half>(bn, epi, a, b, p, grid, st);
}

int gemm_fp8_smem_bytes(int bn) {
  switch (bn) {
    case 16: return Fp8Smem<16>::kBytes;
    case 32: return Fp8Smem<32>::kBytes;
    default: return Fp8Smem<64>::kBytes;
  }
}

void launch_quant_fp8(const void* x, uint8_t* xq, float* sa, int N, int K, int lds, bool bf16, cudaStream_t st) {
  if (bf16)
    launch_k(quant_fp8_kernel<__nv_bfloat16>, dim3(N), dim3(256), 0, st, static_cast<const __nv_bfloat16*>(x), xq, sa,
             K, lds);
  else
    launch_k(quant_fp8_kernel<__half>, dim3(N), dim3(256), 0, st, static_cast<const __half*>(x), xq, sa, K, lds);
}

void launch_rmsnorm_fp8(const float* h, const void* w, uint8_t* xq, float* sa, int N, int H, int lds, float eps,
                        bool bf16, cudaStream_t st) {
  if (bf16)
    launch_k(rmsnorm_fp8_kernel<__nv_bfloat16>, dim3(N), dim3(256), 0, st, h, static_cast<const __nv_bfloat16*>(w), xq,
             sa, H, lds, eps);
  else
    launch_k(rmsnorm_fp8_kernel<__half>, dim3(N), dim3(256), 0, st, h, static_cast<const __half*>(w), xq, sa, H, lds,
             eps);
}

}  // namespace atlas
