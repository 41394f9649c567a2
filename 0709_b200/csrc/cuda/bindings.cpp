// Python bindings of the sm_100a kernels (torch tensors in, launches on the
// current CUDA stream).  Also owns TMA descriptor creation: tensor maps are
// encoded on the host through the driver entry point (no libcuda link) and
// cached per (address, shape, box).

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <torch/extension.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "attention.h"
#include "peer_ring.h"
#include "gemm.h"
#include "gemm_fp8.h"
#include "kernels.h"
#include "tp.h"

namespace {

using atlas::AttnParams;
using atlas::GemmParams;

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e == cudaSuccess && q == cudaDriverEntryPointSuccess) fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  TORCH_CHECK(fn != nullptr, "cuTensorMapEncodeTiled is not available from the CUDA driver");
  return fn;
}

struct MapKey {
  uint64_t ptr;
  uint64_t d[5];
  uint32_t box[5];
  int rank;
  int dtype;
  bool operator==(const MapKey& o) const { return std::memcmp(this, &o, sizeof(MapKey)) == 0; }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    size_t h = std::hash<uint64_t>()(k.ptr);
    for (int i = 0; i < 5; ++i) h = h * 1000003u ^ std::hash<uint64_t>()(k.d[i] * 31 + k.box[i]);
    return h ^ (k.rank * 7 + k.dtype);
  }
};

std::mutex g_map_mu;
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;

CUtensorMapDataType tma_dtype(torch::ScalarType t) {
  if (t == torch::kBFloat16) return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  TORCH_CHECK(t == torch::kHalf, "TMA operands must be fp16 or bf16");
  return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

// Row-major [outer, inner] with row stride `ld` elements; box {128 bytes, box_outer}, 128B swizzle
// (64 elements of fp16/bf16, 128 of fp8).
CUtensorMap map_2d(const torch::Tensor& t, int64_t inner, int64_t outer, int64_t ld, int box_outer) {
  const bool byte = t.element_size() == 1;
  const uint32_t box_inner = byte ? 128 : 64;
  MapKey k{};
  k.ptr = reinterpret_cast<uint64_t>(t.data_ptr());
  k.d[0] = inner;
  k.d[1] = outer;
  k.d[2] = ld;
  k.box[0] = box_inner;
  k.box[1] = box_outer;
  k.rank = 2;
  k.dtype = static_cast<int>(t.scalar_type());
  std::lock_guard<std::mutex> g(g_map_mu);
  auto it = g_maps.find(k);
  if (it != g_maps.end()) return it->second;
  if (g_maps.size() > 8192) g_maps.clear();
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * t.element_size()};
  cuuint32_t box[2] = {box_inner, static_cast<cuuint32_t>(box_outer)};
  cuuint32_t es[2] = {1, 1};
  CUresult r = encode_fn()(&m, byte ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : tma_dtype(t.scalar_type()), 2, t.data_ptr(), dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (2d) failed: ", static_cast<int>(r));
  g_maps.emplace(k, m);
  return m;
}

// KV cache [L, NP, 2, Hkv, ps, hd] as 5-D {hd, ps, Hkv, 2, L*NP}; box {64, ps, 1, 1, 1}.
CUtensorMap map_kv(const torch::Tensor& kv) {
  TORCH_CHECK(kv.dim() == 6 && kv.is_contiguous(), "kv cache must be a contiguous [L, NP, 2, Hkv, ps, hd] tensor");
  const int64_t L = kv.size(0), NP = kv.size(1), Hkv = kv.size(3), ps = kv.size(4), hd = kv.size(5);
  MapKey k{};
  k.ptr = reinterpret_cast<uint64_t>(kv.data_ptr());
  k.d[0] = hd;
  k.d[1] = ps;
  k.d[2] = Hkv;
  k.d[3] = 2;
  k.d[4] = L * NP;
  k.box[0] = 64;
  k.box[1] = static_cast<uint32_t>(ps);
  k.rank = 5;
  k.dtype = static_cast<int>(kv.scalar_type());
  std::lock_guard<std::mutex> g(g_map_mu);
  auto it = g_maps.find(k);
  if (it != g_maps.end()) return it->second;
  CUtensorMap m;
  const int64_t es_b = kv.element_size();
  cuuint64_t dims[5] = {static_cast<cuuint64_t>(hd), static_cast<cuuint64_t>(ps), static_cast<cuuint64_t>(Hkv), 2,
                        static_cast<cuuint64_t>(L * NP)};
  cuuint64_t strides[4] = {static_cast<cuuint64_t>(hd * es_b), static_cast<cuuint64_t>(ps * hd * es_b),
                           static_cast<cuuint64_t>(Hkv * ps * hd * es_b),
                           static_cast<cuuint64_t>(2 * Hkv * ps * hd * es_b)};
  cuuint32_t box[5] = {64, static_cast<cuuint32_t>(ps), 1, 1, 1};
  cuuint32_t es[5] = {1, 1, 1, 1, 1};
  CUresult r = encode_fn()(&m, tma_dtype(kv.scalar_type()), 5, kv.data_ptr(), dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (kv) failed: ", static_cast<int>(r));
  g_maps.emplace(k, m);
  return m;
}

// q [M, Hq, 128] as (128, Hq, M): one box = 64 dimensions x the G query heads of a kv head x the
// 128 / G tokens of a row tile (128 rows of 128 B, 128B-swizzled like the K/V stages).  Not
// cached: a graph captures the map once; an eager call encodes its own (host only, ~1 us).
CUtensorMap map_q(const torch::Tensor& q, int64_t G) {
  TORCH_CHECK(q.dim() == 3 && q.is_contiguous() && q.size(2) == 128, "q must be contiguous [M, Hq, 128]");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(q.data_ptr()) % 16 == 0, "q must be 16-byte aligned");
  const int64_t M = q.size(0), Hq = q.size(1);
  const int64_t es_b = q.element_size();
  CUtensorMap m;
  cuuint64_t dims[3] = {128, static_cast<cuuint64_t>(Hq), static_cast<cuuint64_t>(M)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(128 * es_b), static_cast<cuuint64_t>(Hq * 128 * es_b)};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(G), static_cast<cuuint32_t>(128 / G)};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = encode_fn()(&m, tma_dtype(q.scalar_type()), 3, q.data_ptr(), dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (q) failed: ", static_cast<int>(r));
  return m;
}

int pick_bn(int64_t n) {
  if (n <= 16) return 16;
  if (n <= 32) return 32;
  if (n <= 64) return 64;
  if (n <= 128) return 128;
  return 256;
}

// CTA slots per SM the split-K heuristic fills.  ATLAS_GEMM_CTAS_PER_SM=1 leaves
// half of each SM free so the next kernel (PDL) can become resident and start
// its prologue and weight prefetch while this one drains.
int ctas_per_sm(int bn) {
  static const int cap = [] {
    const char* v = std::getenv("ATLAS_GEMM_CTAS_PER_SM");
    return v != nullptr ? std::max(1, std::atoi(v)) : 2;
  }();
  const int smem = atlas::gemm_smem_bytes(bn) + 1024;
  return std::max(1, std::min(cap, (228 * 1024) / smem));
}

// Split-K factor: fill ~all CTA slots when the tile count alone cannot; a
// function of (M, K, bn) only, so a row's result never depends on batch size
// within one bn bucket.
std::pair<int, int> pick_splits(int64_t M, int64_t N, int64_t K, int bn, int num_sms) {
  const int64_t tiles = ((M + 127) / 128) * ((N + bn - 1) / bn);
  const int64_t kb = (K + 63) / 64;
  const int64_t slots = static_cast<int64_t>(num_sms) * ctas_per_sm(bn);
  int64_t splits = 1;
  if (tiles * 4 < slots * 3) splits = std::max<int64_t>(1, std::min<int64_t>({kb / 2, slots / tiles, 8}));
  // Power-of-two cluster sizes pack into the GPCs without stranded SMs
  // (ATLAS_GEMM_POW2_SPLITS=0 keeps any size).
  static const bool pow2 = [] {
    const char* v = std::getenv("ATLAS_GEMM_POW2_SPLITS");
    return v == nullptr || v[0] != '0';
  }();
  if (pow2) {
    int64_t p = 1;
    while (p * 2 <= splits) p *= 2;
    splits = p;
  }
  int64_t kbps = (kb + splits - 1) / splits;
  splits = (kb + kbps - 1) / kbps;
  return {static_cast<int>(splits), static_cast<int>(kbps)};
}

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

// Load streamed weight tiles with the evict-first L2 policy: weights are read
// once per forward, so they should not displace activations, KV pages and
// split partials (ATLAS_L2_EVICT_FIRST=0 disables).
int stream_hint() {
  static const int v = [] {
    const char* e = std::getenv("ATLAS_L2_EVICT_FIRST");
    return (e == nullptr || e[0] != '0') ? 1 : 0;
  }();
  return v;
}

void check_cuda(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}

// ---------------------------------------------------------------- GEMM
// out = epilogue(x @ w^T).  w [M, K] contiguous; x [N, K] with unit inner stride.
std::vector<int64_t> gemm_impl(const torch::Tensor& w, const torch::Tensor& x, void* out_ptr, int64_t ldo,
                               int64_t epi, const torch::Tensor& err, int64_t force_splits,
                               const atlas::PeerOut* peer, const GemmParams* extra = nullptr) {
  check_cuda(w, "w");
  check_cuda(x, "x");
  TORCH_CHECK(w.dim() == 2 && w.is_contiguous(), "w must be contiguous [M, K]");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "x must be [N, K] with unit inner stride");
  TORCH_CHECK(w.scalar_type() == x.scalar_type(), "w and x must share a dtype");
  const int64_t M = w.size(0), K = w.size(1), N = x.size(0);
  TORCH_CHECK(x.size(1) == K, "x inner dimension mismatch");
  TORCH_CHECK(K % 8 == 0 && x.stride(0) % 8 == 0, "K and the activation row stride must be multiples of 8");
  const int bn = pick_bn(N);
  auto sp = pick_splits(M, N, K, bn, num_sms());
  if (force_splits > 0) {
    const int64_t kb = (K + 63) / 64;
    const int64_t fs = std::min<int64_t>(force_splits, 8);
    int64_t kbps = (kb + fs - 1) / fs;
    sp = {static_cast<int>((kb + kbps - 1) / kbps), static_cast<int>(kbps)};
  }
  if (epi == atlas::kEpiSilu) {
    TORCH_CHECK(M % 128 == 0, "gate/up GEMM needs M % 128 == 0");
  }
  const c10::cuda::CUDAGuard guard(w.device());
  CUtensorMap a = map_2d(w, K, M, K, 128);
  CUtensorMap b = map_2d(x, K, N, x.stride(0), bn);
  GemmParams p{};
  if (extra != nullptr) p = *extra;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.ldo = static_cast<int>(ldo);
  p.splits = sp.first;
  p.kb_per_split = sp.second;
  p.bf16 = w.scalar_type() == torch::kBFloat16;
  p.out = out_ptr;
  p.err = err.data_ptr<int>();
  if (peer != nullptr) p.peer = *peer;
  p.stream_hint = stream_hint();
  atlas::launch_gemm_tn(a, b, p, bn, static_cast<int>(epi), at::cuda::getCurrentCUDAStream());
  return {bn, sp.first, sp.second};
}

std::vector<int64_t> gemm(torch::Tensor w, torch::Tensor x, torch::Tensor out, int64_t epi, torch::Tensor ws,
                          torch::Tensor counters, torch::Tensor err, int64_t force_splits) {
  check_cuda(out, "out");
  TORCH_CHECK(epi != atlas::kEpiPeer, "use gemm_peer for the peer epilogue");
  if (epi == atlas::kEpiResidual || epi == atlas::kEpiF32) {
    TORCH_CHECK(out.scalar_type() == torch::kFloat32, "fp32 output expected for this epilogue");
  } else {
    TORCH_CHECK(out.scalar_type() == w.scalar_type(), "activation-dtype output expected");
  }
  TORCH_CHECK(out.stride(-1) == 1, "out must have unit inner stride");
  return gemm_impl(w, x, out.data_ptr(), out.stride(0), epi, err, force_splits, nullptr);
}

// Row-parallel GEMM whose fp32 output tile is stored into every destination
// (raw device addresses: local or CUDA-IPC-mapped peer buffers, row stride
// `ldo` floats), followed by a release of the incremented local sequence
// number into each destination's flag word.
std::vector<int64_t> gemm_peer(torch::Tensor w, torch::Tensor x, std::vector<int64_t> dst, int64_t ldo,
                               std::vector<int64_t> flags, int64_t ticket, int64_t seq, torch::Tensor ws,
                               torch::Tensor counters, torch::Tensor err, bool sentinel) {
  (void)ws;
  (void)counters;
  TORCH_CHECK(!dst.empty() && dst.size() <= static_cast<size_t>(atlas::kMaxPeers) &&
                  (sentinel || dst.size() == flags.size()),
              "gemm_peer needs 1..8 destinations, one flag each unless in sentinel mode");
  atlas::PeerOut po{};
  po.ndst = static_cast<int>(dst.size());
  po.sentinel = sentinel ? 1 : 0;
  for (size_t i = 0; i < dst.size(); ++i) {
    TORCH_CHECK(dst[i] != 0 && (dst[i] & 3) == 0, "bad peer address");
    po.dst[i] = reinterpret_cast<float*>(dst[i]);
    if (!sentinel) {
      TORCH_CHECK(flags[i] != 0 && (flags[i] & 3) == 0, "bad peer flag address");
      po.flag[i] = reinterpret_cast<uint32_t*>(flags[i]);
    }
  }
  TORCH_CHECK(sentinel || (ticket != 0 && seq != 0), "gemm_peer needs ticket and sequence words");
  po.ticket = reinterpret_cast<uint32_t*>(ticket);
  po.seq = reinterpret_cast<uint32_t*>(seq);
  return gemm_impl(w, x, nullptr, ldo, atlas::kEpiPeer, err, 0, &po);
}

// ----------------------------------------------------------------- fp8
int fp8_pick_bn(int64_t n) { return n <= 16 ? 16 : (n <= 32 ? 32 : 64); }

// Split-K for the fp8 kernel: as for bf16, plus enough splits that one CTA
// covers at most kFp8MaxKbPerCta K blocks (its scales live in shared memory).
std::pair<int, int> fp8_pick_splits(int64_t M, int64_t N, int64_t K, int bn) {
  const int64_t tiles = ((M + 127) / 128) * ((N + bn - 1) / bn);
  const int64_t kb = K / 128;
  int64_t splits = 1;
  const int64_t slots = static_cast<int64_t>(num_sms()) * (bn <= 32 ? 2 : 1);  // CTAs resident per SM
  if (tiles * 4 < slots * 3) splits = std::max<int64_t>(1, std::min<int64_t>({kb / 2, slots / tiles, 8}));
  splits = std::max<int64_t>(splits, (kb + atlas::kFp8MaxKbPerCta - 1) / atlas::kFp8MaxKbPerCta);
  TORCH_CHECK(splits <= 8, "fp8 GEMM: K too long for 8 splits of ", atlas::kFp8MaxKbPerCta, " blocks");
  {  // power-of-two cluster sizes (see pick_splits); round up so the scale table still fits
    int64_t p = 1;
    while (p < splits) p *= 2;
    splits = std::min<int64_t>(p, 8);
  }
  int64_t kbps = (kb + splits - 1) / splits;
  splits = (kb + kbps - 1) / kbps;
  return {static_cast<int>(splits), static_cast<int>(kbps)};
}

std::vector<int64_t> gemm_fp8_impl(const torch::Tensor& wq, const torch::Tensor& sw, const torch::Tensor& xq,
                                   const torch::Tensor& sa, void* out_ptr, int64_t ldo, bool out_bf16, int64_t epi,
                                   const torch::Tensor& err, const atlas::PeerOut* peer) {
  check_cuda(wq, "wq");
  TORCH_CHECK(wq.element_size() == 1 && xq.element_size() == 1, "fp8 operands must be 1-byte tensors");
  TORCH_CHECK(wq.dim() == 2 && wq.is_contiguous() && xq.dim() == 2 && xq.is_contiguous(), "fp8 operand layout");
  const int64_t M = wq.size(0), K = wq.size(1), N = xq.size(0);
  TORCH_CHECK(xq.size(1) == K && K % 128 == 0, "fp8 GEMM needs K % 128 == 0 and matching operands");
  TORCH_CHECK(sw.scalar_type() == torch::kFloat32 && sw.is_contiguous() && sw.size(0) == (M + 127) / 128 &&
                  sw.size(1) == K / 128, "weight scales must be fp32 [ceil(M/128), K/128]");
  TORCH_CHECK(sa.scalar_type() == torch::kFloat32 && sa.is_contiguous() && sa.size(0) == K / 128 && sa.size(1) >= N,
              "activation scales must be fp32 [K/128, >= N]");
  if (epi == atlas::kEpiSilu) TORCH_CHECK(M % 128 == 0, "gate/up GEMM needs M % 128 == 0");
  const int bn = fp8_pick_bn(N);
  auto sp = fp8_pick_splits(M, N, K, bn);
  const c10::cuda::CUDAGuard guard(wq.device());
  CUtensorMap a = map_2d(wq, K, M, K, 128);
  CUtensorMap b = map_2d(xq, K, N, K, bn);
  atlas::Fp8GemmParams p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.ldo = static_cast<int>(ldo);
  p.splits = sp.first;
  p.kb_per_split = sp.second;
  p.out_bf16 = out_bf16 ? 1 : 0;
  p.lds = static_cast<int>(sa.size(1));
  p.sw = sw.data_ptr<float>();
  p.sa = sa.data_ptr<float>();
  p.out = out_ptr;
  p.err = err.data_ptr<int>();
  if (peer != nullptr) p.peer = *peer;
  p.stream_hint = stream_hint();
  atlas::launch_gemm_fp8(a, b, p, bn, static_cast<int>(epi), at::cuda::getCurrentCUDAStream());
  return {bn, sp.first, sp.second};
}

std::vector<int64_t> gemm_fp8(torch::Tensor wq, torch::Tensor sw, torch::Tensor xq, torch::Tensor sa,
                              torch::Tensor out, int64_t epi, torch::Tensor err) {
  check_cuda(out, "out");
  TORCH_CHECK(epi != atlas::kEpiPeer, "use gemm_fp8_peer for the peer epilogue");
  const bool f32 = epi == atlas::kEpiResidual || epi == atlas::kEpiF32;
  TORCH_CHECK(f32 ? out.scalar_type() == torch::kFloat32
                  : (out.scalar_type() == torch::kBFloat16 || out.scalar_type() == torch::kHalf),
              "output dtype does not match the epilogue");
  TORCH_CHECK(out.stride(-1) == 1, "out must have unit inner stride");
  return gemm_fp8_impl(wq, sw, xq, sa, out.data_ptr(), out.stride(0), out.scalar_type() == torch::kBFloat16, epi,
                       err, nullptr);
}

std::vector<int64_t> gemm_fp8_peer(torch::Tensor wq, torch::Tensor sw, torch::Tensor xq, torch::Tensor sa,
                                   std::vector<int64_t> dst, int64_t ldo, std::vector<int64_t> flags, int64_t ticket,
                                   int64_t seq, torch::Tensor err) {
  TORCH_CHECK(!dst.empty() && dst.size() <= static_cast<size_t>(atlas::kMaxPeers) && dst.size() == flags.size(),
              "gemm_fp8_peer needs 1..8 destinations, one flag each");
  atlas::PeerOut po{};
  po.ndst = static_cast<int>(dst.size());
  for (size_t i = 0; i < dst.size(); ++i) {
    po.dst[i] = reinterpret_cast<float*>(dst[i]);
    po.flag[i] = reinterpret_cast<uint32_t*>(flags[i]);
  }
  po.ticket = reinterpret_cast<uint32_t*>(ticket);
  po.seq = reinterpret_cast<uint32_t*>(seq);
  return gemm_fp8_impl(wq, sw, xq, sa, nullptr, ldo, false, atlas::kEpiPeer, err, &po);
}

void quant_fp8(torch::Tensor x, torch::Tensor xq, torch::Tensor sa) {
  TORCH_CHECK(x.is_contiguous() && xq.is_contiguous() && x.dim() == 2 && x.size(1) % 128 == 0, "quant_fp8 layout");
  TORCH_CHECK(sa.size(0) == x.size(1) / 128 && sa.size(1) >= x.size(0), "quant_fp8 scale layout");
  const c10::cuda::CUDAGuard guard(x.device());
  atlas::launch_quant_fp8(x.data_ptr(), static_cast<uint8_t*>(xq.data_ptr()), sa.data_ptr<float>(),
                          static_cast<int>(x.size(0)), static_cast<int>(x.size(1)), static_cast<int>(sa.size(1)),
                          x.scalar_type() == torch::kBFloat16, at::cuda::getCurrentCUDAStream());
}

void rmsnorm_fp8(torch::Tensor h, torch::Tensor w, torch::Tensor xq, torch::Tensor sa, double eps) {
  TORCH_CHECK(h.scalar_type() == torch::kFloat32 && h.is_contiguous() && h.size(1) % 128 == 0, "rmsnorm_fp8 input");
  TORCH_CHECK(sa.size(0) == h.size(1) / 128 && sa.size(1) >= h.size(0), "rmsnorm_fp8 scale layout");
  const c10::cuda::CUDAGuard guard(h.device());
  atlas::launch_rmsnorm_fp8(h.data_ptr<float>(), w.data_ptr(), static_cast<uint8_t*>(xq.data_ptr()),
                            sa.data_ptr<float>(), static_cast<int>(h.size(0)), static_cast<int>(h.size(1)),
                            static_cast<int>(sa.size(1)), static_cast<float>(eps), w.scalar_type() == torch::kBFloat16,
                            at::cuda::getCurrentCUDAStream());
}

// --------------------------------------------- GEMM with folded RMSNorm
// One entry for the epilogues that fold RMSNorm and RoPE into the GEMM:
//   nin_ss (optional) [K / 128, ld]: per-tile sums of h^2 -> column scale rstd;
//   kEpiResidualNorm: out = h (fp32, += acc), hb = h in the activation dtype,
//     nout_ss [M / 128, ld] receives this GEMM's per-tile sums of h^2;
//   kEpiRope: q_out / kv_layer receive the rotated q/k heads and the v heads.
std::vector<int64_t> gemm_fused(torch::Tensor w, torch::Tensor x, c10::optional<torch::Tensor> out, int64_t epi,
                                torch::Tensor err, c10::optional<torch::Tensor> nin_ss, double eps,
                                c10::optional<torch::Tensor> nout_ss, c10::optional<torch::Tensor> hb,
                                c10::optional<torch::Tensor> table, c10::optional<torch::Tensor> pos,
                                c10::optional<torch::Tensor> slots, c10::optional<torch::Tensor> kv_layer,
                                c10::optional<torch::Tensor> q_out, int64_t Hq, int64_t Hkv) {
  const int64_t M = w.size(0), K = w.size(1), N = x.size(0);
  GemmParams ex{};
  if (nin_ss.has_value()) {
    TORCH_CHECK(nin_ss->scalar_type() == torch::kFloat32 && nin_ss->is_contiguous() && nin_ss->dim() == 2 &&
                    nin_ss->size(0) * 128 == K && nin_ss->size(1) >= N,
                "nin_ss must be fp32 [K / 128, >= N]");
    ex.nin.ss = nin_ss->data_ptr<float>();
    ex.nin.tiles = static_cast<int>(nin_ss->size(0));
    ex.nin.ld = static_cast<int>(nin_ss->size(1));
    ex.nin.inv_h = 1.0f / static_cast<float>(K);
    ex.nin.eps = static_cast<float>(eps);
  }
  void* out_ptr = nullptr;
  int64_t ldo = 0;
  if (epi == atlas::kEpiResidualNorm) {
    TORCH_CHECK(out.has_value() && nout_ss.has_value() && hb.has_value(), "residual-norm epilogue needs h, hb, ss");
    TORCH_CHECK(out->scalar_type() == torch::kFloat32 && out->is_contiguous() && out->size(1) == M, "h layout");
    TORCH_CHECK(hb->scalar_type() == w.scalar_type() && hb->is_contiguous() && hb->size(1) == M, "hb layout");
    TORCH_CHECK(M % 128 == 0 && nout_ss->scalar_type() == torch::kFloat32 && nout_ss->is_contiguous() &&
                    nout_ss->size(0) * 128 == M && nout_ss->size(1) >= N,
                "nout_ss must be fp32 [M / 128, >= N]");
    ex.nout.ss = nout_ss->data_ptr<float>();
    ex.nout.ld = static_cast<int>(nout_ss->size(1));
    ex.nout.hb = hb->data_ptr();
    out_ptr = out->data_ptr();
    ldo = out->stride(0);
  } else if (epi == atlas::kEpiRope) {
    TORCH_CHECK(table.has_value() && pos.has_value() && slots.has_value() && kv_layer.has_value() &&
                    q_out.has_value(), "rope epilogue needs table, positions, slots, kv layer and q output");
    TORCH_CHECK(kv_layer->dim() == 5 && kv_layer->size(4) == 128 && kv_layer->is_contiguous() &&
                    kv_layer->size(2) == Hkv && kv_layer->scalar_type() == w.scalar_type(),
                "kv layer must be [pages, 2, Hkv, ps, 128] in the activation dtype");
    TORCH_CHECK(M == (Hq + 2 * Hkv) * 128 && q_out->is_contiguous() && q_out->numel() >= N * Hq * 128,
                "rope epilogue: M must be (Hq + 2 Hkv) * 128");
    TORCH_CHECK(pos->scalar_type() == torch::kInt32 && slots->scalar_type() == torch::kInt32 &&
                    table->scalar_type() == torch::kFloat32 && table->size(1) == 128, "rope input dtypes");
    ex.rope.table = table->data_ptr<float>();
    ex.rope.pos = pos->data_ptr<int>();
    ex.rope.slots = slots->data_ptr<int>();
    ex.rope.kv = kv_layer->data_ptr();
    ex.rope.q = q_out->data_ptr();
    ex.rope.Hq = static_cast<int>(Hq);
    ex.rope.Hkv = static_cast<int>(Hkv);
    ex.rope.ps = static_cast<int>(kv_layer->size(3));
    ex.rope.num_pages = static_cast<int>(kv_layer->size(0));
    ex.rope.max_pos = static_cast<int>(table->size(0));
  } else {
    TORCH_CHECK(epi == atlas::kEpiStore || epi == atlas::kEpiSilu || epi == atlas::kEpiF32,
                "gemm_fused: store, SiLU, fp32, residual-norm or rope epilogue");
    TORCH_CHECK(out.has_value() && out->stride(-1) == 1, "out must have unit inner stride");
    TORCH_CHECK((epi == atlas::kEpiF32) == (out->scalar_type() == torch::kFloat32), "output dtype vs epilogue");
    out_ptr = out->data_ptr();
    ldo = out->stride(0);
  }
  return gemm_impl(w, x, out_ptr, ldo, epi, err, 0, nullptr, &ex);
}

// Embedding gather that also writes the activation-dtype copy and the
// per-128-feature sums of h^2 that the first folded-norm GEMM needs.
void embed_norm(torch::Tensor tok, torch::Tensor table, torch::Tensor h, torch::Tensor hb, torch::Tensor ss,
                torch::Tensor err) {
  TORCH_CHECK(tok.scalar_type() == torch::kInt32 && h.scalar_type() == torch::kFloat32, "embed dtypes");
  TORCH_CHECK(table.size(1) % 128 == 0 && ss.size(0) * 128 == table.size(1) && ss.size(1) >= tok.numel(),
              "ss must be fp32 [H / 128, >= M]");
  const c10::cuda::CUDAGuard guard(h.device());
  atlas::launch_embed_norm(tok.data_ptr<int>(), table.data_ptr(), h.data_ptr<float>(), hb.data_ptr(),
                           ss.data_ptr<float>(), static_cast<int>(ss.size(1)), static_cast<int>(tok.numel()),
                           static_cast<int>(table.size(1)), static_cast<int>(table.size(0)),
                           table.scalar_type() == torch::kBFloat16, err.data_ptr<int>(),
                           at::cuda::getCurrentCUDAStream());
}

// --------------------------------------------------- tensor parallelism
void tp_reduce_rmsnorm(int64_t recv, int64_t slot_stride, int64_t flags, int64_t seq, int64_t nsrc, torch::Tensor h,
                       c10::optional<torch::Tensor> gamma, c10::optional<torch::Tensor> x, double eps,
                       torch::Tensor err, bool sentinel) {
  TORCH_CHECK(h.scalar_type() == torch::kFloat32 && h.is_contiguous() && h.dim() == 2, "h must be contiguous fp32");
  const int64_t M = h.size(0), H = h.size(1);
  TORCH_CHECK(H % 32 == 0 && H <= 16384 && recv != 0 && (recv & 15) == 0 && slot_stride % 4 == 0,
              "reduce layout: H must be a multiple of 32 and at most 16384");
  TORCH_CHECK(nsrc >= 1 && nsrc <= atlas::kMaxPeers, "1..8 sources");
  TORCH_CHECK(gamma.has_value() == x.has_value(), "gamma and x go together");
  bool bf16 = false;
  if (x.has_value()) {
    TORCH_CHECK(x->is_contiguous() && x->size(0) == M && x->size(1) == H, "x shape");
    TORCH_CHECK(gamma->scalar_type() == x->scalar_type(), "gamma/x dtype");
    bf16 = x->scalar_type() == torch::kBFloat16;
  }
  const c10::cuda::CUDAGuard guard(h.device());
  atlas::launch_tp_reduce_rmsnorm(reinterpret_cast<const float*>(recv), slot_stride,
                                  reinterpret_cast<const uint32_t*>(flags), reinterpret_cast<const uint32_t*>(seq),
                                  static_cast<int>(nsrc), sentinel ? 1 : 0, h.data_ptr<float>(),
                                  gamma.has_value() ? gamma->data_ptr() : nullptr,
                                  x.has_value() ? x->data_ptr() : nullptr, static_cast<int>(M), static_cast<int>(H),
                                  static_cast<float>(eps), bf16, err.data_ptr<int>(), at::cuda::getCurrentCUDAStream());
}

void tp_wait(int64_t flags, int64_t seq, int64_t nsrc, torch::Tensor err) {
  const c10::cuda::CUDAGuard guard(err.device());
  atlas::launch_tp_wait(reinterpret_cast<const uint32_t*>(flags), reinterpret_cast<const uint32_t*>(seq),
                        static_cast<int>(nsrc), err.data_ptr<int>(), at::cuda::getCurrentCUDAStream());
}

// Wall-time limit of the cross-GPU waits (tp_reduce_rmsnorm, tp_wait) on one device.
void set_peer_wait_ns(int64_t ns, int64_t device) {
  TORCH_CHECK(ns > 0, "the peer wait limit must be positive");
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  const cudaError_t e = atlas::set_peer_wait_ns(static_cast<uint64_t>(ns));
  TORCH_CHECK(e == cudaSuccess, "set_peer_wait_ns: ", cudaGetErrorString(e));
}

int64_t peer_wait_ns(int64_t device) {
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  uint64_t ns = 0;
  const cudaError_t e = atlas::get_peer_wait_ns(&ns);
  TORCH_CHECK(e == cudaSuccess, "peer_wait_ns: ", cudaGetErrorString(e));
  return static_cast<int64_t>(ns);
}

// ------------------------------------------------------- peer rings
// ring_push: src (device or pinned host address) holds header + payload.
void ring_push(int64_t src, int64_t bytes, int64_t peer_ring, int64_t seq, int64_t device) {
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  const cudaError_t e = atlas::launch_ring_push(reinterpret_cast<const void*>(src), bytes,
                                                reinterpret_cast<void*>(peer_ring), static_cast<uint32_t>(seq),
                                                at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(e == cudaSuccess, "ring_push: ", cudaGetErrorString(e));
}

// ring_pop: dst (device or pinned host address) receives header + payload;
// nbytes_out (int32 device tensor) the payload length or -1; err the ring's flag.
void ring_pop(int64_t ring, int64_t seq, int64_t dst, int64_t dst_bytes, torch::Tensor nbytes_out, torch::Tensor err,
              int64_t limit_ns) {
  const c10::cuda::CUDAGuard guard(err.device());
  TORCH_CHECK(err.scalar_type() == torch::kInt32 && nbytes_out.scalar_type() == torch::kInt32, "int32 flags");
  const cudaError_t e = atlas::launch_ring_pop(reinterpret_cast<const void*>(ring), static_cast<uint32_t>(seq),
                                               reinterpret_cast<void*>(dst), dst_bytes, nbytes_out.data_ptr<int>(),
                                               err.data_ptr<int>(), static_cast<uint64_t>(limit_ns),
                                               at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(e == cudaSuccess, "ring_pop: ", cudaGetErrorString(e));
}

// CUDA IPC: a plain cudaMalloc region (not the caching allocator, whose blocks
// share one IPC handle per segment) that peers map into their address space.
int64_t ipc_malloc(int64_t bytes, int64_t device) {
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  void* p = nullptr;
  TORCH_CHECK(cudaMalloc(&p, static_cast<size_t>(bytes)) == cudaSuccess, "cudaMalloc of the symmetric buffer failed");
  TORCH_CHECK(cudaMemset(p, 0, static_cast<size_t>(bytes)) == cudaSuccess, "cudaMemset failed");
  return reinterpret_cast<int64_t>(p);
}

void ipc_free(int64_t ptr, int64_t device) {
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  cudaFree(reinterpret_cast<void*>(ptr));
}

py::bytes ipc_handle(int64_t ptr, int64_t device) {
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(ptr));
  TORCH_CHECK(e == cudaSuccess, "cudaIpcGetMemHandle failed: ", cudaGetErrorString(e));
  return py::bytes(reinterpret_cast<const char*>(&h), sizeof(h));
}

int64_t ipc_open(py::bytes handle, int64_t device) {
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  std::string s = handle;
  TORCH_CHECK(s.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, s.data(), sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  TORCH_CHECK(e == cudaSuccess, "cudaIpcOpenMemHandle failed: ", cudaGetErrorString(e));
  return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t ptr, int64_t device) {
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr));
}

bool can_access_peer(int64_t device, int64_t peer) {
  int ok = 0;
  cudaDeviceCanAccessPeer(&ok, static_cast<int>(device), static_cast<int>(peer));
  return ok != 0;
}

// View raw device memory owned elsewhere (a symmetric buffer) as a tensor.
torch::Tensor wrap_ptr(int64_t ptr, std::vector<int64_t> sizes, torch::ScalarType dtype, int64_t device) {
  auto opts = torch::TensorOptions().dtype(dtype).device(torch::kCUDA, static_cast<c10::DeviceIndex>(device));
  return torch::from_blob(reinterpret_cast<void*>(ptr), sizes, [](void*) {}, opts);
}

// ----------------------------------------------------------- attention
// The grid is sized for the longest context a graph may see; on a short one
// the surplus splits find no pages and exit instead of each paying the CTA's
// fixed cost for a single chunk (ATLAS_ATTN_MIN_PAGES overrides, default 4).
static int attn_min_pages() {
  static const int min_pages = [] {
    const char* v = std::getenv("ATLAS_ATTN_MIN_PAGES");
    return v != nullptr ? std::max(1, std::atoi(v)) : 4;
  }();
  return min_pages;
}

void attention(torch::Tensor q, torch::Tensor kv, int64_t layer, torch::Tensor out, torch::Tensor dparams,
               torch::Tensor prefix_pages, torch::Tensor row_full, torch::Tensor row_len, torch::Tensor row_mask,
               torch::Tensor tail_pages, torch::Tensor part_o, torch::Tensor part_ml, torch::Tensor err,
               int64_t splits, bool run_tc, bool run_combine, bool direct_out, double scale, bool fused_merge) {
  check_cuda(q, "q");
  TORCH_CHECK(q.dim() == 3 && q.size(2) == 128 && q.is_contiguous(), "q must be contiguous [M, Hq, 128]");
  TORCH_CHECK(kv.scalar_type() == q.scalar_type(), "q and kv dtype mismatch");
  TORCH_CHECK(kv.size(5) == 128 && kv.size(4) % 8 == 0 && 64 % kv.size(4) == 0,
              "kernels need head_dim 128 and a page size dividing 64 that is a multiple of 8");
  TORCH_CHECK(row_mask.dim() == 2 && row_mask.scalar_type() == torch::kInt64, "row_mask must be int64 [M, W]");
  TORCH_CHECK(tail_pages.dim() == 2, "tail_pages must be [M, T]");
  const int64_t M = q.size(0), Hq = q.size(1), Hkv = kv.size(3);
  TORCH_CHECK(Hq % Hkv == 0, "Hq must be a multiple of Hkv");
  const int64_t G = Hq / Hkv;
  TORCH_CHECK(128 % G == 0, "GQA group must divide 128");
  if (fused_merge) {
    TORCH_CHECK(run_tc && run_combine && !direct_out, "the fused merge runs both stages and writes the output");
    TORCH_CHECK(splits >= 1 && splits <= atlas::attention_max_cluster(q.scalar_type() == torch::kBFloat16),
                "fused-merge splits must fit one cluster");
  } else if (!direct_out && run_tc) {
    TORCH_CHECK(part_o.numel() >= splits * M * Hq * 128 && part_ml.numel() >= splits * M * Hq * 2,
                "attention split workspace too small");
  }
  const c10::cuda::CUDAGuard guard(q.device());
  CUtensorMap kvmap{}, qmap{};
  if (run_tc) {
    kvmap = map_kv(kv);
    qmap = map_q(q, G);
  }
  AttnParams p{};
  p.q = q.data_ptr();
  p.kv = kv.data_ptr();
  p.out = out.data_ptr();
  p.dparams = dparams.data_ptr<int>();
  p.prefix_pages = prefix_pages.data_ptr<int>();
  p.row_full = row_full.data_ptr<int>();
  p.row_len = row_len.data_ptr<int>();
  p.row_mask = row_mask.data_ptr<int64_t>();
  p.tail_pages = tail_pages.data_ptr<int>();
  p.part_o = part_o.numel() ? part_o.data_ptr<float>() : nullptr;
  p.part_ml = part_ml.numel() ? reinterpret_cast<float2*>(part_ml.data_ptr<float>()) : nullptr;
  p.err = err.data_ptr<int>();
  p.M = static_cast<int>(M);
  p.Hq = static_cast<int>(Hq);
  p.Hkv = static_cast<int>(Hkv);
  p.page_size = static_cast<int>(kv.size(4));
  p.num_pages = static_cast<int>(kv.size(1));
  p.layer = static_cast<int>(layer);
  p.mask_words = static_cast<int>(row_mask.size(1));
  p.tail_stride = static_cast<int>(tail_pages.size(1));
  p.splits = run_tc ? static_cast<int>(splits) : 0;
  p.direct_out = direct_out ? 1 : 0;
  p.bf16 = q.scalar_type() == torch::kBFloat16;
  p.min_pages_per_split = attn_min_pages();
  p.fused_merge = fused_merge ? 1 : 0;
  p.scale = static_cast<float>(scale);
  const int row_tiles = static_cast<int>((M * G + 127) / 128);
  atlas::launch_attention(kvmap, qmap, p, run_tc, run_combine, row_tiles, at::cuda::getCurrentCUDAStream());
}

// Device -> pinned host copy on the current stream, with no allocator bookkeeping: safe to
// capture into a CUDA graph (the graph then copies into the same host buffer on every replay).
void copy_to_host_async(torch::Tensor host, torch::Tensor src) {
  TORCH_CHECK(src.is_cuda() && src.is_contiguous(), "source must be a contiguous CUDA tensor");
  TORCH_CHECK(!host.is_cuda() && host.is_pinned() && host.is_contiguous(), "destination must be pinned host memory");
  TORCH_CHECK(host.nbytes() >= src.nbytes(), "destination smaller than the source");
  const c10::cuda::CUDAGuard guard(src.device());
  C10_CUDA_CHECK(cudaMemcpyAsync(host.data_ptr(), src.data_ptr(), src.nbytes(), cudaMemcpyDeviceToHost,
                                 at::cuda::getCurrentCUDAStream()));
}

// Pinned host -> device copy on the current stream, then `event` (a cudaEvent_t handle, 0 for
// none) recorded after it: one call for the static batch's per-forward input copy and the
// event that guards the reuse of its host buffer.
void upload_async(torch::Tensor dev, torch::Tensor host, int64_t event) {
  TORCH_CHECK(dev.is_cuda() && dev.is_contiguous(), "destination must be a contiguous CUDA tensor");
  TORCH_CHECK(!host.is_cuda() && host.is_pinned() && host.is_contiguous(), "source must be pinned host memory");
  TORCH_CHECK(dev.nbytes() >= host.nbytes(), "destination smaller than the source");
  const c10::cuda::CUDAGuard guard(dev.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  C10_CUDA_CHECK(cudaMemcpyAsync(dev.data_ptr(), host.data_ptr(), host.nbytes(), cudaMemcpyHostToDevice, st));
  if (event != 0) C10_CUDA_CHECK(cudaEventRecord(reinterpret_cast<cudaEvent_t>(event), st));
}

// --------------------------------------------------------- elementwise
void embed(torch::Tensor tok, torch::Tensor table, torch::Tensor out, torch::Tensor err) {
  TORCH_CHECK(tok.scalar_type() == torch::kInt32 && out.scalar_type() == torch::kFloat32, "embed dtypes");
  const c10::cuda::CUDAGuard guard(out.device());
  atlas::launch_embed(tok.data_ptr<int>(), table.data_ptr(), out.data_ptr<float>(), static_cast<int>(tok.numel()),
                      static_cast<int>(table.size(1)), static_cast<int>(table.size(0)),
                      table.scalar_type() == torch::kBFloat16, err.data_ptr<int>(), at::cuda::getCurrentCUDAStream());
}

void rmsnorm(torch::Tensor x, torch::Tensor w, torch::Tensor out, double eps) {
  TORCH_CHECK(x.scalar_type() == torch::kFloat32 && x.is_contiguous() && x.size(1) % 4 == 0, "rmsnorm input");
  const c10::cuda::CUDAGuard guard(x.device());
  atlas::launch_rmsnorm(x.data_ptr<float>(), w.data_ptr(), out.data_ptr(), static_cast<int>(x.size(0)),
                        static_cast<int>(x.size(1)), static_cast<float>(eps), w.scalar_type() == torch::kBFloat16,
                        at::cuda::getCurrentCUDAStream());
}

void rope_append(torch::Tensor qkv, torch::Tensor table, torch::Tensor pos, torch::Tensor slots, torch::Tensor kv_layer,
                 torch::Tensor qout, int64_t Hq, int64_t Hkv, torch::Tensor err) {
  TORCH_CHECK(qkv.is_contiguous() && kv_layer.is_contiguous() && qout.is_contiguous(), "rope_append contiguity");
  const c10::cuda::CUDAGuard guard(qkv.device());
  const int hd = static_cast<int>(kv_layer.size(4));
  atlas::launch_rope_append(qkv.data_ptr(), table.data_ptr<float>(), pos.data_ptr<int>(), slots.data_ptr<int>(),
                            kv_layer.data_ptr(), qout.data_ptr(), static_cast<int>(qkv.size(0)), static_cast<int>(Hq),
                            static_cast<int>(Hkv), hd, static_cast<int>(kv_layer.size(3)),
                            static_cast<int>(kv_layer.size(0)), static_cast<int>(table.size(0)),
                            qkv.scalar_type() == torch::kBFloat16, err.data_ptr<int>(),
                            at::cuda::getCurrentCUDAStream());
}

void kv_copy_pages(torch::Tensor kv, torch::Tensor plan, torch::Tensor err) {
  TORCH_CHECK(plan.scalar_type() == torch::kInt32 && plan.dim() == 2 && plan.size(1) == 3, "plan must be int32 [n,3]");
  const c10::cuda::CUDAGuard guard(kv.device());
  atlas::launch_kv_copy_pages(kv.data_ptr(), plan.data_ptr<int>(), static_cast<int>(plan.size(0)),
                              static_cast<int>(kv.size(0)), static_cast<int>(kv.size(1)), static_cast<int>(kv.size(3)),
                              static_cast<int>(kv.size(4)), static_cast<int>(kv.size(5)), err.data_ptr<int>(),
                              at::cuda::getCurrentCUDAStream());
}

// plan int32 [max_n, 3] and count int32 [1] on the device (read when the kernel runs).
void kv_copy_pages_counted(torch::Tensor kv, torch::Tensor plan, torch::Tensor count, torch::Tensor err) {
  TORCH_CHECK(plan.scalar_type() == torch::kInt32 && plan.dim() == 2 && plan.size(1) == 3, "plan must be int32 [n,3]");
  TORCH_CHECK(count.scalar_type() == torch::kInt32 && count.numel() >= 1 && count.is_cuda(), "count must be int32");
  const c10::cuda::CUDAGuard guard(kv.device());
  atlas::launch_kv_copy_pages_counted(kv.data_ptr(), plan.data_ptr<int>(), count.data_ptr<int>(),
                                      static_cast<int>(plan.size(0)), static_cast<int>(kv.size(0)),
                                      static_cast<int>(kv.size(1)), static_cast<int>(kv.size(3)),
                                      static_cast<int>(kv.size(4)), static_cast<int>(kv.size(5)), err.data_ptr<int>(),
                                      at::cuda::getCurrentCUDAStream());
}

void kv_move_slots(torch::Tensor kv, torch::Tensor src, torch::Tensor dst, torch::Tensor err) {
  TORCH_CHECK(src.numel() == dst.numel() && src.numel() <= 64, "at most 64 slot moves per launch");
  const c10::cuda::CUDAGuard guard(kv.device());
  atlas::launch_kv_move_slots(kv.data_ptr(), src.data_ptr<int>(), dst.data_ptr<int>(), static_cast<int>(src.numel()),
                              static_cast<int>(kv.size(0)), static_cast<int>(kv.size(1)), static_cast<int>(kv.size(3)),
                              static_cast<int>(kv.size(4)), static_cast<int>(kv.size(5)), err.data_ptr<int>(),
                              at::cuda::getCurrentCUDAStream());
}

void topk(torch::Tensor logits, int64_t k, c10::optional<torch::Tensor> keys, double inv_temp, torch::Tensor out_lp,
          torch::Tensor out_id) {
  TORCH_CHECK(logits.scalar_type() == torch::kFloat32 && logits.is_contiguous(), "logits must be contiguous fp32");
  TORCH_CHECK(k >= 1 && k <= 8, "top-k supports 1 <= k <= 8");
  const c10::cuda::CUDAGuard guard(logits.device());
  const int64_t B = logits.size(0), V = logits.size(1);
  // Enough vocabulary chunks to spread the scan over every SM (<= 256 chunks, >= 1024 entries each).
  const int chunks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(
      {256, (V + 1023) / 1024, (2 * num_sms() + B - 1) / B})));
  auto part = torch::empty({B * chunks * atlas::topk_record_floats()}, logits.options());
  atlas::launch_topk(logits.data_ptr<float>(), static_cast<int>(B), static_cast<int>(V), static_cast<int>(k),
                     keys.has_value() ? keys->data_ptr<int64_t>() : nullptr, static_cast<float>(inv_temp),
                     out_lp.data_ptr<float>(), out_id.data_ptr<int64_t>(), part.data_ptr<float>(), chunks,
                     at::cuda::getCurrentCUDAStream());
}

void gather_logprobs(torch::Tensor logits, torch::Tensor rows, torch::Tensor toks, torch::Tensor lse, torch::Tensor out,
                     torch::Tensor err) {
  TORCH_CHECK(logits.scalar_type() == torch::kFloat32 && logits.is_contiguous(), "logits must be contiguous fp32");
  const c10::cuda::CUDAGuard guard(logits.device());
  atlas::launch_gather_logprobs(logits.data_ptr<float>(), static_cast<int>(logits.size(0)),
                                static_cast<int>(logits.size(1)), rows.data_ptr<int>(), toks.data_ptr<int>(),
                                static_cast<int>(rows.numel()), lse.data_ptr<float>(), out.data_ptr<float>(),
                                err.data_ptr<int>(), at::cuda::getCurrentCUDAStream());
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels: tcgen05/TMA GEMM and paged attention, fused norm/rope/append, KV copies, top-k";
  m.def("gemm", &gemm, "tcgen05 GEMM out = epi(x @ w^T); returns [bn, splits, kb_per_split]");
  m.def("attention", &attention, "paged attention (tensor-core shared range + per-row tail/combine)");
  m.def("set_attention_phase_buffer", [](torch::Tensor buf) {
    TORCH_CHECK(!buf.defined() || buf.numel() == 0 || (buf.is_cuda() && buf.scalar_type() == torch::kInt64),
                "phase buffer must be a CUDA int64 tensor (or empty to switch off)");
    atlas::set_attention_phase_buffer(buf.defined() && buf.numel() ? reinterpret_cast<unsigned long long*>(
                                                                          buf.data_ptr<int64_t>())
                                                                    : nullptr);
  }, "profiling: SM-clock stamps of the tensor-core attention kernel's steps into buf (empty: off)");
  m.def("attention_max_cluster", [](bool bf16) { return atlas::attention_max_cluster(bf16); },
        "largest split cluster of the fused-merge attention on the current device");
  m.def("embed", &embed);
  m.def("rmsnorm", &rmsnorm);
  m.def("rope_append", &rope_append);
  m.def("kv_copy_pages", &kv_copy_pages);
  m.def("kv_copy_pages_counted", &kv_copy_pages_counted,
        "copy-on-write pages whose plan and count are read on the device (capturable once for any count)");
  m.def("kv_move_slots", &kv_move_slots);
  m.def("upload_async", &upload_async, "pinned host -> device copy on the current stream, then an event record");
  m.def("copy_to_host_async", &copy_to_host_async, "device -> pinned host copy on the current stream (capturable)");
  m.def("topk", &topk);
  m.def("gather_logprobs", &gather_logprobs);
  m.def("gemm_fused", &gemm_fused, "GEMM with folded RMSNorm (residual-norm / rope / scaled epilogues)");
  m.def("embed_norm", &embed_norm);
  m.attr("EPI_RESIDUAL_NORM") = static_cast<int>(atlas::kEpiResidualNorm);
  m.attr("EPI_ROPE") = static_cast<int>(atlas::kEpiRope);
  m.def("gemm_peer", &gemm_peer, "tcgen05 GEMM with the fp32 tile stored into peer buffers, then a release flag");
  m.def("tp_reduce_rmsnorm", &tp_reduce_rmsnorm, "wait for peers, h += sum of partials, x = rmsnorm(h)");
  m.def("tp_wait", &tp_wait);
  m.def("ring_push", &ring_push, "copy a message into a peer GPU's ring and publish its sequence number");
  m.def("ring_pop", &ring_pop, "bounded wait for a ring's next message, then copy it out");
  m.def("set_peer_wait_ns", &set_peer_wait_ns, "wall-time limit (ns) of cross-GPU waits on a device");
  m.def("peer_wait_ns", &peer_wait_ns);
  m.def("gemm_fp8", &gemm_fp8, "block-scaled fp8 tcgen05 GEMM; returns [bn, splits, kb_per_split]");
  m.def("gemm_fp8_peer", &gemm_fp8_peer);
  m.def("quant_fp8", &quant_fp8, "per-token 1x128 e4m3 quantization");
  m.def("rmsnorm_fp8", &rmsnorm_fp8, "RMSNorm straight to e4m3 + 1x128 scales");
  m.def("ipc_malloc", &ipc_malloc);
  m.def("ipc_free", &ipc_free);
  m.def("ipc_handle", &ipc_handle);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
  m.def("can_access_peer", &can_access_peer);
  m.def("wrap_ptr", &wrap_ptr);
  m.attr("EPI_STORE") = static_cast<int>(atlas::kEpiStore);
  m.attr("EPI_RESIDUAL") = static_cast<int>(atlas::kEpiResidual);
  m.attr("EPI_SILU") = static_cast<int>(atlas::kEpiSilu);
  m.attr("EPI_F32") = static_cast<int>(atlas::kEpiF32);
  m.attr("EPI_PEER") = static_cast<int>(atlas::kEpiPeer);
}
