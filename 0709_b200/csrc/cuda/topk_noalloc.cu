// Allocation-free variant of the vocabulary top-k (see topk_noalloc.h for who
// needs it and the calling contract).  No counterpart in the reference
// implementation.
//
// It runs the same two kernels as the regular binding (launch_topk: one block
// per vocabulary chunk of a row, then one warp per row merging the chunk
// records); only the scratch for the chunk records differs -- here it is the
// fixed device array below instead of a per-call allocation.

#include <cstdio>
#include <mutex>

#include "kernels.h"
#include "topk_noalloc.h"

namespace {
constexpr int kMaxRecords = 4096;  // (row, chunk) records
constexpr int kRecordFloatsMax = 26;  // must cover topk_record_floats()
constexpr int kMaxDevices = 64;
}  // namespace

// Fixed scratch for the chunk records: 4096 x 26 floats = 416 KiB per GPU.
// In host code this name is only a stand-in for the symbol; the device address
// comes from cudaGetSymbolAddress below.
static __device__ __align__(256) float atlas_topk_scratch[kMaxRecords * kRecordFloatsMax];

namespace {
std::mutex g_mu;
float* g_scratch_ptr[kMaxDevices] = {};
int g_num_sms[kMaxDevices] = {};

// Once per device, with that device current: resolve the array's device address.
int setup(int dev, float** ptr, int* sms) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, atlas_topk_scratch);
    if (e != cudaSuccess || p == nullptr) {
      std::fprintf(stderr, "atlas_topk_logprobs_noalloc: cudaGetSymbolAddress failed on device %d: %s\n", dev,
                   cudaGetErrorString(e));
      return ATLAS_NOALLOC_ECUDA;
    }
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess || n <= 0) {
      std::fprintf(stderr, "atlas_topk_logprobs_noalloc: cannot read the SM count of device %d\n", dev);
      return ATLAS_NOALLOC_ECUDA;
    }
    g_scratch_ptr[dev] = static_cast<float*>(p);
    g_num_sms[dev] = n;
  }
  *ptr = g_scratch_ptr[dev];
  *sms = g_num_sms[dev];
  return ATLAS_NOALLOC_OK;
}
}  // namespace

extern "C" int atlas_topk_logprobs_noalloc(const float* logits, int rows, int vocab, int k, const int64_t* keys,
                                           float inv_temperature, float* out_logprobs, int64_t* out_ids,
                                           cudaStream_t stream) {
  if (logits == nullptr || out_logprobs == nullptr || out_ids == nullptr || rows < 1 || vocab < 1 || k < 1 || k > 8) {
    std::fprintf(stderr, "atlas_topk_logprobs_noalloc: invalid argument (rows=%d vocab=%d k=%d)\n", rows, vocab, k);
    return ATLAS_NOALLOC_EINVAL;
  }
  const int rec_floats = atlas::topk_record_floats();
  if (rec_floats > kRecordFloatsMax) {
    std::fprintf(stderr,
                 "atlas_topk_logprobs_noalloc: the kernel's chunk record (%d floats) is larger than the fixed "
                 "scratch's record slot (%d floats); the library was built inconsistently\n",
                 rec_floats, kRecordFloatsMax);
    return ATLAS_NOALLOC_ECUDA;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return ATLAS_NOALLOC_ECUDA;
  float* scratch = nullptr;
  int sms = 0;
  const int rc = setup(dev, &scratch, &sms);
  if (rc != ATLAS_NOALLOC_OK) return rc;
  // Same vocabulary split as the regular binding: enough chunks to spread a
  // row over the SMs, at most 256 chunks of at least 1024 entries.
  long long chunks = (vocab + 1023LL) / 1024;
  chunks = chunks < 256 ? chunks : 256;
  const long long by_sms = (2LL * sms + rows - 1) / rows;
  chunks = chunks < by_sms ? chunks : by_sms;
  if (chunks < 1) chunks = 1;
  const long long records = static_cast<long long>(rows) * chunks;
  if (records > kMaxRecords) {
    std::fprintf(stderr,
                 "atlas_topk_logprobs_noalloc: %d rows x %lld vocabulary chunks = %lld records exceed the fixed "
                 "scratch of %d records; split the call into fewer rows\n",
                 rows, chunks, records, kMaxRecords);
    return ATLAS_NOALLOC_ETOOLARGE;
  }
  // The launches' own return codes: an error left earlier by the caller stays the caller's to read.
  const cudaError_t e = atlas::launch_topk(logits, rows, vocab, k, keys, inv_temperature, out_logprobs, out_ids,
                                           scratch, static_cast<int>(chunks), stream);
  if (e != cudaSuccess) {
    std::fprintf(stderr, "atlas_topk_logprobs_noalloc: launch failed: %s\n", cudaGetErrorString(e));
    return ATLAS_NOALLOC_ECUDA;
  }
  return ATLAS_NOALLOC_OK;
}
