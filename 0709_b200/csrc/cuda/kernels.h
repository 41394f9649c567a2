// Launch wrappers of the CUDA-core kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace atlas {

void launch_embed(const int* tok, const void* table, float* out, int M, int H, int V, bool bf16, int* err,
                  cudaStream_t st);
void launch_embed_norm(const int* tok, const void* table, float* h, void* hb, float* ss, int ss_ld, int M, int H, int V,
                       bool bf16, int* err, cudaStream_t st);
void launch_rmsnorm(const float* x, const void* w, void* out, int M, int H, float eps, bool bf16, cudaStream_t st);
void launch_rope_append(const void* qkv, const float* table, const int* pos, const int* slots, void* kv_layer,
                        void* qout, int M, int Hq, int Hkv, int hd, int ps, int num_pages, int max_pos, bool bf16,
                        int* err, cudaStream_t st);
void launch_kv_copy_pages_counted(void* kv, const int* plan, const int* count, int max_n, int layers, int num_pages,
                                  int Hkv, int ps, int hd, int* err, cudaStream_t st);
void launch_kv_copy_pages(void* kv, const int* plan, int n, int layers, int num_pages, int Hkv, int ps, int hd,
                          int* err, cudaStream_t st);
void launch_kv_move_slots(void* kv, const int* src, const int* dst, int n, int layers, int num_pages, int Hkv, int ps,
                          int hd, int* err, cudaStream_t st);
cudaError_t launch_topk(const float* logits, int B, int V, int k, const int64_t* keys, float inv_temp, float* out_lp,
                 int64_t* out_id, float* part, int chunks, cudaStream_t st);
int topk_record_floats();
void launch_gather_logprobs(const float* logits, int R, int V, const int* rows, const int* toks, int n, float* lse,
                            float* out, int* err, cudaStream_t st);

}  // namespace atlas
