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
// floats of the chunk-partial buffer the multi-row attention path needs for R rows
int attn_part_floats(int R, int H, int D, int max_seq);
// one row: 8-CTA clusters merging through distributed shared memory; several rows:
// partial CTAs + combine through `part` (attn_part_floats(R, ...) floats); shared_rows:
// the rows belong to one sequence (prefill) and read the same chunks
int launch_attention(const float *q, const float *kc, const float *vc, float *part, int8_t *out_q, float *out_f,
                     const int32_t *row_seq, const int32_t *row_i, const int32_t *cache_pos, int layer, int n_layers,
                     int R, int H, int KVH, int D, int max_seq, int *err, cudaStream_t s, bool shared_rows = false);
int launch_swiglu(const float *y, int8_t *out_q, float *out_f, int R, int F, cudaStream_t s);
int lmhead_grid(int dev);
int launch_lmhead(const float *xn, const float *W, float *logits, float2 *cand, int32_t *tok, float2 *pairs,
                  int idx0, int R, int hidden, int vocab, int grid, cudaStream_t s);
int launch_merge_argmax(const float2 *pairs, int world, int R, int32_t *tok, cudaStream_t s);
int launch_dequant_residual(const int32_t *C, const float *scales, const float *offsets, float *x, int R, int N,
                            cudaStream_t s);
int launch_advance(int32_t *cache_pos, const int32_t *seqs, int nseq, int n, cudaStream_t s);

// model internals shared with the weight-file readers (q35_model.cu, q35_ingest.cu)
const q35_model_config &model_config(q35_model m);
int model_set_embeddings_rm(q35_model m, const float *embed_rm, const float *final_norm, const float *lm_head);

// tensor-parallel communicator (q35_tp.cu)
int tp_allreduce_i32(q35_tp t, int32_t *buf, size_t count, cudaStream_t s);
int tp_allgather(q35_tp t, const void *send, void *recv, size_t bytes, cudaStream_t s);
int tp_rank(q35_tp t);
int tp_buffer(q35_tp t, int slot, size_t bytes, void **out);
void tp_attach(q35_tp t, int delta);
int tp_world(q35_tp t);
// all-reduce of the int32 partials C (n = rows x N), then x += dequant(C): a one-shot
// exchange over NVLink peer memory when every rank mapped every peer, else NCCL
int tp_allreduce_dequant(q35_tp t, int32_t *C, int64_t n, int32_t N, const float *scales, const float *offsets,
                         float *x, int *err, cudaStream_t s);
// R rows (up to 64): the same exchange, then RMSNorm of the new rows with norm_w (int8 into q
// and/or fp32 into out), bit-identical to launch_rmsnorm after tp_allreduce_dequant;
// *fused is false (nothing launched) when the peer-memory path is not available for this size
int tp_allreduce_dequant_norm(q35_tp t, int32_t *C, int32_t R, int32_t N, const float *scales, const float *offsets,
                              float *x, const float *norm_w, float eps, int8_t *q, float *out, int *err, cudaStream_t s,
                              bool *fused);

}  // namespace q35
