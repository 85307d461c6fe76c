// q35_layer.cuh -- launchers of the layer/model kernels (q35_layer.cu)
#pragma once
#include "q35_internal.cuh"

namespace q35 {

int launch_embed(const int32_t *ids, const float *E, float *x, int R, int hidden, int vocab, int *err,
                 cudaStream_t s);
int launch_rmsnorm(const float *x, const float *w, float *out, int8_t *q, int R, int dim, float eps,
                   cudaStream_t s);
int launch_rope_kv(const float *yqkv, float *q, float *kc, float *vc, const int32_t *row_seq,
                   const int32_t *row_i, const int32_t *cache_pos, const float2 *cs, int layer,
                   int n_layers, int R, int H, int KVH, int D, int max_seq, int rope_mode, int *err,
                   cudaStream_t s);
int attn_part_floats(int R, int H, int D, int max_seq);
int launch_attention(const float *q, const float *kc, const float *vc, float *part, int8_t *out_q,
                     float *out_f, const int32_t *row_seq, const int32_t *row_i, const int32_t *cache_pos,
                     int layer, int n_layers, int R, int H, int KVH, int D, int max_seq, cudaStream_t s);
int launch_swiglu(const float *y, int8_t *out_q, float *out_f, int R, int F, cudaStream_t s);
int lmhead_grid(int dev);
int launch_lmhead(const float *xn, const float *W, float *logits, float2 *cand, int32_t *tok, int R,
                  int hidden, int vocab, int grid, cudaStream_t s);
int launch_advance(int32_t *cache_pos, const int32_t *seqs, int nseq, int n, cudaStream_t s);

}  // namespace q35
