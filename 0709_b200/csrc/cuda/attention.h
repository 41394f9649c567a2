// Host/device interface of the paged attention kernels (head_dim 128).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace atlas {

struct AttnParams {
  const void* q;         // [M, Hq, 128] rotated queries
  const void* kv;        // cache [L, pages, 2, Hkv, page_size, 128]
  void* out;             // [M, Hq, 128]
  const int* dparams;    // device scalars: shared_len, n_shared_pages, mask_base
  const int* prefix_pages;
  const int* row_full;   // [M]
  const int* row_len;    // [M]
  const int64_t* row_mask;  // [M, mask_words]
  const int* tail_pages;    // [M, tail_stride]
  float* part_o;         // [splits, M, Hq, 128]
  float2* part_ml;       // [splits, M, Hq] (running max in log2 units, sum)
  int* err;
  int M, Hq, Hkv, page_size, num_pages, layer;
  int mask_words, tail_stride, splits, direct_out, bf16;
  int min_pages_per_split;  // a split covers at least this many pages (surplus splits exit at once)
  int fused_merge;          // 1: the splits of a head form one cluster and merge + tail in the same kernel
  float scale;
  // Profiling only (null otherwise): per CTA of the tensor-core kernel, kAttnPhases SM-clock
  // stamps of its pipeline steps (see attn_shared_tc) and the global timer at entry.
  unsigned long long* phases;
};

constexpr int kAttnPhases = 20;

// Phase buffer for the next launches of the tensor-core attention kernel (nullptr: off).
void set_attention_phase_buffer(unsigned long long* buf);

// Largest cluster (splits of one head) the fused-merge path may launch with on this device: 16 when the
// device can hold a 16-CTA cluster of the tensor-core kernel, else 8.
int attention_max_cluster(bool bf16);

// kvmap: the cache (see map_kv); qmap: q [M, Hq, 128] as a 3-D map (128, Hq, M) with box
// (64, Hq / Hkv, 128 / (Hq / Hkv)) and 128B swizzle, one box per 64-dimension half of a tile.
void launch_attention(const CUtensorMap& kvmap, const CUtensorMap& qmap, const AttnParams& p, bool run_tc,
                      bool run_combine, int row_tiles, cudaStream_t st);

}  // namespace atlas
