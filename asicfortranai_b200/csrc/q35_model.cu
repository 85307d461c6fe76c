// q35_model.cu -- LLaMA model runtime on one GPU: llama_model.f90 (init_llama_model,
// forward_llama, cleanup_llama_model), transformer_layer.f90 (apply_transformer_layer
// with the weights-allocated branches) and the generation loop of llama_generate.f90
// (greedy by default; temperature, top-k and top-p sampling of sampling.f90 on request).
//
// Per layer, R rows (a prompt's positions, or one position of each decoded sequence):
//   rmsnorm(x)->int8 | q|k|v GEMV | RoPE + KV-cache write | attention -> int8 |
//   o GEMV, epilogue x += y | rmsnorm->int8 | gate|up GEMV (+ SwiGLU -> int8 in its
//   epilogue at <= 4 rows, a separate kernel after the tensor cores) | down GEMV,
//   epilogue x += y
// then final rmsnorm, fp32 LM head and the next token (greedy argmax or the sampler).
// q|k|v and gate|up are each one matrix (q|k|v columns concatenated, gate/up columns
// interleaved): quantization is per column and both consume the same int8 activations,
// so the fused matmul returns exactly the three (two) results.  Under tensor parallelism
// o and down produce int32 partials that the exchange sums, dequantizes and adds to x; at
// one row the exchange also forms the next RMSNorm.
// Sequence positions and the current tokens live on the device, so a decode step is
// position-independent and is captured once as a CUDA graph.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "q35_layer.cuh"

using namespace q35;

namespace {

struct LayerW {
    q35_weights qkv = nullptr, o = nullptr, gu = nullptr, d = nullptr;
    float *attn_norm = nullptr, *ffn_norm = nullptr;
};

}  // namespace

struct q35_model_s {
    q35_ctx ctx = nullptr;
    q35_model_config cfg{};
    q35_tp tp = nullptr;                 // tensor-parallel group (nullptr: one GPU)
    int rank = 0, world = 1;
    // local (per-rank) sizes: H, KVH, F, V are the shard's; Hg.. the model's
    int H = 0, KVH = 0, D = 0, hidden = 0, F = 0, V = 0, L = 0, QN = 0, KN = 0, B = 0, maxR = 0;
    int Hg = 0, KVHg = 0, Fg = 0, Vg = 0;
    std::vector<LayerW> layers;
    float *embed = nullptr, *final_norm = nullptr, *lm_head = nullptr;
    float2 *rope = nullptr;
    float *kc = nullptr, *vc = nullptr;
    int32_t *cache_pos = nullptr;        // [B] device
    std::vector<int32_t> host_pos;       // mirror of cache_pos
    // activations [maxR][...]
    float *x = nullptr, *yqkv = nullptr, *q = nullptr, *ygu = nullptr, *xn = nullptr, *logits = nullptr;
    int32_t *cacc = nullptr;             // row-split matmul partial sums [maxR][hidden] (TP)
    float2 *pairs = nullptr;             // greedy candidates of this rank [maxR]
    float2 *pairs_all = nullptr;         // gathered candidates [world][maxR]
    float *logits_all = nullptr;         // gathered logits [world][maxR][V] (TP, on request)
    int8_t *xi8 = nullptr;
    int8_t *hq = nullptr;                // SwiGLU output, the down projection's int8 input [maxR][F]
    float *apart = nullptr;              // attention chunk partials, several-row path [64][H][chunks][D+2]
    float2 *cand = nullptr;
    int32_t *tok = nullptr;              // [B] current token of each sequence
    int32_t *tok_tmp = nullptr;          // [maxR] greedy tokens of a prefill's LM rows
    int32_t *ids = nullptr, *row_seq = nullptr, *row_i = nullptr, *seqs = nullptr;
    int32_t *hist = nullptr;             // [max_steps][B] tokens recorded by decode steps
    int32_t *step_ctr = nullptr;
    int32_t *draws = nullptr;            // [B] sampled tokens so far per sequence (draw counters)
    q35_sampling samp{};                 // next-token rule (mode 0: greedy)
    int max_steps = 0;
    bool rows_one_seq = false;           // the rows of the current forward share one sequence
    int lm_grid = 0;
    // decode step graph (B rows, one per sequence)
    cudaGraph_t g = nullptr;
    cudaGraphExec_t gexec = nullptr;
    bool gather_logits = false;          // decode graph also gathers the logits (TP)
    std::vector<void *> allocs;
};

namespace {

template <typename T>
int dalloc(q35_model m, T **p, size_t n) {
    *p = nullptr;
    if (n == 0) n = 1;
    cudaError_t e = cudaMalloc(reinterpret_cast<void **>(p), n * sizeof(T));
    if (e != cudaSuccess) return set_error(Q35_ERR_NOMEM, std::string("model allocation: ") + cudaGetErrorString(e));
    m->allocs.push_back(*p);
    return Q35_OK;
}

int check_cfg(const q35_model_config &c) {
    if (c.n_layers < 1 || c.hidden < 32 || c.n_heads < 1 || c.n_kv_heads < 1 || c.head_dim < 32 ||
        c.ffn < 2 || c.vocab < 1 || c.max_seq < 1 || c.max_batch < 1)
        return set_error(Q35_ERR_INVALID, "model config: non-positive or too small dimension");
    if (c.hidden % 32 || (c.ffn & 1))
        return set_error(Q35_ERR_INVALID, "model config: hidden must be a multiple of 32, ffn even");
    if (c.head_dim != 128 && c.head_dim != 256)
        return set_error(Q35_ERR_INVALID, "model config: head_dim must be 128 or 256");
    if (c.n_heads % c.n_kv_heads)
        return set_error(Q35_ERR_INVALID, "model config: n_heads must be a multiple of n_kv_heads");
    if (c.wformat != Q35_FMT_3P5BIT && c.wformat != Q35_FMT_INT4)
        return set_error(Q35_ERR_INVALID, "model config: unknown weight format");
    if (c.max_seq > 8192) return set_error(Q35_ERR_INVALID, "model config: max_seq above 8192");
    if (c.head_dim == 256 && c.max_seq > 4096)
        return set_error(Q35_ERR_INVALID, "model config: head_dim 256 supports max_seq up to 4096");
    if (c.rope_mode != 0 && c.rope_mode != 1) return set_error(Q35_ERR_INVALID, "model config: rope_mode 0 or 1");
    return Q35_OK;
}

// transformer_layer.f90:96-118 (frequency table) and the cos/sin of :195-196, computed
// on the host with the C library in binary32, as the reference does
void rope_table(const q35_model_config &c, std::vector<float2> &t) {
    const int half = c.head_dim / 2;
    t.resize((size_t)c.max_seq * half);
    for (int d = 0; d < half; ++d) {
        const float e = (-2.0f * (float)d) / (float)c.head_dim;
        const float th = powf(c.rope_theta, e);
        for (int p = 0; p < c.max_seq; ++p) {
            const float f = (float)p * th;
            t[(size_t)p * half + d] = make_float2(cosf(f), sinf(f));
        }
    }
}

// reference-layout bytes of several matrices with the same K, columns concatenated
void concat_cols(const std::vector<const int8_t *> &src, const std::vector<int> &ncols, int K,
                 std::vector<int8_t> &dst) {
    size_t total = 0;
    for (int n : ncols) total += (size_t)n;
    dst.resize(total * (K / 2));
    size_t off = 0;
    for (size_t i = 0; i < src.size(); ++i) {
        std::memcpy(dst.data() + off, src[i], (size_t)ncols[i] * (K / 2));
        off += (size_t)ncols[i] * (K / 2);
    }
}

void concat_f(const std::vector<const float *> &src, const std::vector<int> &n, std::vector<float> &dst) {
    dst.clear();
    for (size_t i = 0; i < src.size(); ++i) dst.insert(dst.end(), src[i], src[i] + n[i]);
}

int upload_matrix(q35_model m, q35_weights *slot, int fmt, const int8_t *wq, const float *s, const float *o,
                  int N, int K) {
    if (*slot) { q35_weights_free(*slot); *slot = nullptr; }
    q35_weights h = nullptr;
    int st = weights_alloc(m->ctx, fmt, N, K, &h);
    if (!st) st = weights_fill(m->ctx, h, wq, s, o, 0);
    if (!st) {
        cudaError_t e = cudaStreamSynchronize(m->ctx->stream);
        if (e != cudaSuccess) st = set_error(Q35_ERR_CUDA, cudaGetErrorString(e));
    }
    if (st) { if (h) q35_weights_free(h); return st; }
    *slot = h;
    return Q35_OK;
}

int generate_matrix(q35_model m, q35_weights *slot, int fmt, int N, int K, uint64_t seed, uint64_t tid,
                    double sigma) {
    if (*slot) { q35_weights_free(*slot); *slot = nullptr; }
    // q35_weights_generate takes the context lock itself
    return q35_weights_generate(m->ctx, fmt, N, K, seed, tid, sigma, slot);
}

// attention of R rows in chunks of 64 rows (the partial buffer holds 64 rows)
int attention_rows(q35_model m, int l, int R) {
    int st = Q35_OK;
    for (int r0 = 0; r0 < R && !st; r0 += 64) {
        const int n = std::min(64, R - r0);
        st = launch_attention(m->q + (size_t)r0 * m->QN, m->kc, m->vc, m->apart, m->xi8 + (size_t)r0 * m->QN, nullptr,
                              m->row_seq + r0, m->row_i + r0, m->cache_pos, l, m->L, n, m->H, m->KVH, m->D,
                              m->cfg.max_seq, m->ctx->ws.err, m->ctx->stream, m->rows_one_seq);
    }
    return st;
}

// one decoder layer over R rows (apply_transformer_layer, transformer_layer.f90:527-565).
// One GPU: o and down add their dequantized output to x in the matmul epilogue.
// Tensor parallel: o and down (row-split) produce int32 partial sums, all-reduced, then
// dequantized and added to x.
//
// Under tensor parallelism at one row, the exchange after o also forms the ffn
// RMSNorm, and the exchange after down the next norm (next_w: the next layer's attn_norm
// into xi8, or the final norm into xn), in one kernel (tp_allreduce_dequant_norm);
// pre_normed says xi8 already holds this layer's attn_norm input, *next_normed that the
// next norm is done.
int layer_rows(q35_model m, int l, int R, bool pre_normed = false, const float *next_w = nullptr,
               int8_t *next_q = nullptr, float *next_out = nullptr, bool *next_normed = nullptr) {
    const q35_model_config &c = m->cfg;
    cudaStream_t s = m->ctx->stream;
    q35_ctx ctx = m->ctx;
    int *err = ctx->ws.err;
    const LayerW &w = m->layers[l];
    if (next_normed) *next_normed = false;
    int st = pre_normed ? Q35_OK : launch_rmsnorm(m->x, w.attn_norm, nullptr, m->xi8, R, m->hidden, c.rms_eps, s);
    // q|k|v: RoPE and the KV-cache writes in the matmul's epilogue (CUDA-core engine), or
    // the separate kernel after the tensor cores
    GemvRope rope;
    rope.q = m->q; rope.kc = m->kc; rope.vc = m->vc;
    rope.row_seq = m->row_seq; rope.row_i = m->row_i; rope.cache_pos = m->cache_pos; rope.cs = m->rope;
    rope.layer = l; rope.n_layers = m->L; rope.H = m->H; rope.KVH = m->KVH; rope.D = m->D;
    rope.max_seq = c.max_seq; rope.rope_mode = c.rope_mode;
    bool roped = false;
    if (!st) st = gemm_rows_rope(ctx, w.qkv, m->xi8, R, m->yqkv, rope, &roped);
    if (!st && !roped) st = gemm_rows(ctx, w.qkv, m->xi8, R, nullptr, m->yqkv, nullptr);
    if (!st && !roped)
        st = launch_rope_kv(m->yqkv, m->q, m->kc, m->vc, m->row_seq, m->row_i, m->cache_pos, m->rope, l, m->L, R,
                            m->H, m->KVH, m->D, c.max_seq, c.rope_mode, err, s);
    if (!st) st = attention_rows(m, l, R);
    bool ffn_normed = false;
    if (m->world == 1) {
        if (!st) st = gemm_rows(ctx, w.o, m->xi8, R, nullptr, m->x, m->x);
    } else {
        if (!st) st = gemm_rows(ctx, w.o, m->xi8, R, m->cacc, nullptr, nullptr);
        if (!st && R == 1)   // (at one row only, as the down exchange in forward_rows)
            st = tp_allreduce_dequant_norm(m->tp, m->cacc, R, m->hidden, w.o->w.scales, w.o->w.offsets, m->x,
                                           w.ffn_norm, c.rms_eps, m->xi8, nullptr, err, s, &ffn_normed);
        if (!st && !ffn_normed)
            st = tp_allreduce_dequant(m->tp, m->cacc, (int64_t)R * m->hidden, m->hidden, w.o->w.scales,
                                      w.o->w.offsets, m->x, err, s);
    }
    if (!st && !ffn_normed) st = launch_rmsnorm(m->x, w.ffn_norm, nullptr, m->xi8, R, m->hidden, c.rms_eps, s);
    // gate|up with SwiGLU and the down projection's int8 quantization in the matmul's
    // epilogue (the CUDA-core engine), or the separate SwiGLU kernel after the tensor cores
    if (!st) st = gemm_rows_swiglu(ctx, w.gu, m->xi8, R, m->ygu, m->hq);
    if (m->world == 1) {
        if (!st) st = gemm_rows(ctx, w.d, m->hq, R, nullptr, m->x, m->x);
    } else {
        bool done = false;
        if (!st) st = gemm_rows(ctx, w.d, m->hq, R, m->cacc, nullptr, nullptr);
        if (!st && next_w)
            st = tp_allreduce_dequant_norm(m->tp, m->cacc, R, m->hidden, w.d->w.scales, w.d->w.offsets, m->x, next_w,
                                           c.rms_eps, next_q, next_out, err, s, &done);
        if (!st && !done)
            st = tp_allreduce_dequant(m->tp, m->cacc, (int64_t)R * m->hidden, m->hidden, w.d->w.scales,
                                      w.d->w.offsets, m->x, err, s);
        if (next_normed) *next_normed = done;
    }
    return st;
}

// final norm + LM head + greedy over rows [lm_r0, lm_r0 + lm_rows); the tokens go to
// tok_dst (replicated on every rank); with gather_logits the full logits of those rows
// end in logits_all ([world][rows][V_local]) on every rank.  With a sampling mode the
// rows from samp_first on are sampled instead (every rank draws the same token from the
// same gathered logits).
int lmhead_rows(q35_model m, int lm_r0, int lm_rows, int32_t *tok_dst, bool gather_logits, int samp_first,
                bool normed = false) {
    const q35_model_config &c = m->cfg;
    cudaStream_t s = m->ctx->stream;
    int st = normed ? Q35_OK
                    : launch_rmsnorm(m->x + (size_t)lm_r0 * m->hidden, m->final_norm, m->xn, nullptr, lm_rows,
                                     m->hidden, c.rms_eps, s);
    const int idx0 = m->rank * m->V;
    for (int r0 = 0; r0 < lm_rows && !st; r0 += 64) {
        const int n = std::min(64, lm_rows - r0);
        st = launch_lmhead(m->xn + (size_t)r0 * m->hidden, m->lm_head, m->logits + (size_t)r0 * m->V, m->cand,
                           m->world == 1 ? tok_dst + r0 : nullptr, m->pairs + r0, idx0, n, m->hidden, m->V,
                           m->lm_grid, s);
    }
    if (!st && m->world > 1) {
        st = tp_allgather(m->tp, m->pairs, m->pairs_all, sizeof(float2) * lm_rows, s);
        if (!st) st = launch_merge_argmax(m->pairs_all, m->world, lm_rows, tok_dst, s);
    }
    const bool sampling = m->samp.mode != Q35_SAMPLE_GREEDY;
    if (!st && (gather_logits || sampling) && m->world > 1)
        st = tp_allgather(m->tp, m->logits, m->logits_all, sizeof(float) * (size_t)lm_rows * m->V, s);
    if (!st && sampling && samp_first < lm_rows) {
        SampleRows a;
        a.logits = m->world == 1 ? m->logits : m->logits_all;
        a.Vl = m->V;
        a.Rtot = lm_rows;
        a.V = m->Vg;
        a.row0 = samp_first;
        a.rows = lm_rows - samp_first;
        a.mode = m->samp.mode;
        a.temperature = m->samp.temperature;
        a.top_k = m->samp.top_k;
        a.top_p = m->samp.top_p;
        a.seed = m->samp.seed;
        a.row_seq = m->row_seq;
        a.row_seq0 = lm_r0;
        a.draws = m->draws;
        a.tokens = tok_dst + samp_first;
        st = launch_sample(a, s);
    }
    return st;
}

// one forward over R rows already described in ids/row_seq/row_i; the LM head runs on
// the rows [lm_r0, lm_r0 + lm_rows) of the final hidden state and writes their next
// tokens to tok_dst (sampled from row samp_first on); afterwards the positions of the
// nseq sequences in `seqs` advance by adv
int forward_rows(q35_model m, int R, int lm_r0, int lm_rows, int32_t *tok_dst, int nseq, int adv,
                 bool gather_logits, int samp_first) {
    cudaStream_t s = m->ctx->stream;
    m->rows_one_seq = nseq < R;   // prefill: the rows share a sequence (and its cache chunks)
    int st = launch_embed(m->ids, m->embed, m->x, R, m->hidden, m->Vg, m->ctx->ws.err, s);
    // under tensor parallelism, at one row, each down exchange also forms the next norm (the
    // next layer's attn_norm into xi8; after the last layer the final norm into xn, when the
    // LM head takes every row) (tp_allreduce_dequant_norm).  The fused kernel takes up to 64
    // rows, but at decode batches its 32 CTAs measured far slower than the exchange and the
    // norm's own grid (TP=2, batch 16: 646 against 865 tok/s)
    const bool fuse = m->world > 1 && R == 1;
    bool pre = false;
    for (int l = 0; l < m->L && !st; ++l) {
        const bool last = l + 1 == m->L;
        bool next = false;
        if (fuse && (!last || (lm_r0 == 0 && lm_rows == R)))
            st = layer_rows(m, l, R, pre, last ? m->final_norm : m->layers[l + 1].attn_norm,
                            last ? nullptr : m->xi8, last ? m->xn : nullptr, &next);
        else
            st = layer_rows(m, l, R, pre);
        pre = next;
    }
    if (!st) st = lmhead_rows(m, lm_r0, lm_rows, tok_dst, gather_logits, samp_first, pre);
    if (!st) st = launch_advance(m->cache_pos, m->seqs, nseq, adv, s);
    return st;
}

// copy the logits of `rows` LM rows to a host (rows, vocab) column-major array
int logits_to_host(q35_model m, int rows, float *host) {
    cudaStream_t s = m->ctx->stream;
    const float *src = m->world == 1 ? m->logits : m->logits_all;
    std::vector<float> t((size_t)m->world * rows * m->V);
    Q35_CUDA_TRY(cudaMemcpyAsync(t.data(), src, t.size() * sizeof(float), cudaMemcpyDeviceToHost, s));
    Q35_CUDA_TRY(cudaStreamSynchronize(s));
    for (int w = 0; w < m->world; ++w)
        for (int i = 0; i < rows; ++i)
            for (int64_t jl = 0; jl < m->V; ++jl)
                host[i + (size_t)rows * ((int64_t)w * m->V + jl)] = t[((size_t)w * rows + i) * m->V + jl];
    return Q35_OK;
}

int check_ready(q35_model m) {
    if (!m) return set_error(Q35_ERR_INVALID, "model is NULL");
    for (const LayerW &w : m->layers)
        if (!w.qkv || !w.o || !w.gu || !w.d) return set_error(Q35_ERR_STATE, "model: layer weights not set");
    return Q35_OK;
}

// first node of the decode-step graph: row r is sequence r at offset 0 of the call, and
// its input token is the sequence's current token (a prefill in between rewrites the row
// tables, so the step sets them itself)
__global__ void decode_rows_kernel(const int32_t *tok, int32_t *ids, int32_t *row_seq, int32_t *row_i,
                                   int32_t *seqs, int B) {
    for (int r = threadIdx.x; r < B; r += blockDim.x) {
        ids[r] = tok[r];
        row_seq[r] = r;
        row_i[r] = 0;
        seqs[r] = r;
    }
}

__global__ void record_kernel(const int32_t *tok, int32_t *hist, int32_t *ctr, int B, int max_steps) {
    const int t = threadIdx.x;
    const int step = *ctr;
    if (step >= 0 && step < max_steps && t < B) hist[(size_t)step * B + t] = tok[t];
    __syncthreads();
    if (t == 0) *ctr = step + 1;
}

}  // namespace

namespace q35 {

const q35_model_config &model_config(q35_model m) { return m->cfg; }

// embeddings [vocab][hidden] row-major, output_weights(hidden, vocab) column-major (that is
// [vocab][hidden] row-major; this rank's rows are kept), final_norm[hidden]; any may be NULL
int model_set_embeddings_rm(q35_model m, const float *embed_rm, const float *final_norm, const float *lm_head) {
    if (!m) return set_error(Q35_ERR_INVALID, "model is NULL");
    DeviceGuard g(m->ctx->device);
    cudaError_t e = cudaSuccess;
    if (embed_rm) e = cudaMemcpy(m->embed, embed_rm, sizeof(float) * (size_t)m->Vg * m->hidden, cudaMemcpyHostToDevice);
    if (e == cudaSuccess && lm_head)
        e = cudaMemcpy(m->lm_head, lm_head + (size_t)m->rank * m->V * m->hidden,
                       sizeof(float) * (size_t)m->V * m->hidden, cudaMemcpyHostToDevice);
    if (e == cudaSuccess && final_norm)
        e = cudaMemcpy(m->final_norm, final_norm, sizeof(float) * m->hidden, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return set_error(Q35_ERR_CUDA, cudaGetErrorString(e));
    return Q35_OK;
}

}  // namespace q35

extern "C" {

int q35_model_create(q35_ctx ctx, const q35_model_config *cfg, q35_model *out) {
    return q35_model_create_tp(ctx, cfg, nullptr, out);
}

int q35_model_create_tp(q35_ctx ctx, const q35_model_config *cfg, q35_tp tp, q35_model *out) {
    if (!ctx || !cfg || !out) return set_error(Q35_ERR_INVALID, "NULL argument");
    *out = nullptr;
    int st = check_cfg(*cfg);
    if (st) return st;
    const int world = tp_world(tp), rank = tp_rank(tp);
    if (cfg->n_heads % world || cfg->n_kv_heads % world || cfg->ffn % (2 * world) || cfg->vocab % world)
        return set_error(Q35_ERR_INVALID, "model config: n_heads, n_kv_heads, ffn/2 and vocab must divide by the TP size");
    DeviceGuard g(ctx->device);
    q35_model m = new q35_model_s();
    m->ctx = ctx;
    m->cfg = *cfg;
    m->tp = tp;
    tp_attach(tp, 1);
    m->world = world;
    m->rank = rank;
    m->Hg = cfg->n_heads; m->KVHg = cfg->n_kv_heads; m->Fg = cfg->ffn; m->Vg = cfg->vocab;
    m->H = cfg->n_heads / world; m->KVH = cfg->n_kv_heads / world; m->D = cfg->head_dim; m->hidden = cfg->hidden;
    m->F = cfg->ffn / world; m->V = cfg->vocab / world; m->L = cfg->n_layers; m->B = cfg->max_batch;
    m->QN = m->H * m->D; m->KN = m->KVH * m->D;
    m->maxR = std::max(cfg->max_batch, cfg->max_seq);
    m->max_steps = cfg->max_seq;
    m->layers.resize(m->L);
    const size_t R = (size_t)m->maxR;
    const size_t widest = (size_t)std::max({m->hidden, m->QN, m->F});
    const size_t kv = (size_t)m->B * m->L * m->KVH * cfg->max_seq * m->D;
    std::vector<float2> rt;
    rope_table(*cfg, rt);
    st = dalloc(m, &m->kc, kv);
    if (!st) st = dalloc(m, &m->vc, kv);
    if (!st) st = dalloc(m, &m->rope, rt.size());
    if (!st) st = dalloc(m, &m->cache_pos, (size_t)m->B);
    if (!st) st = dalloc(m, &m->x, R * m->hidden);
    if (!st) st = dalloc(m, &m->yqkv, R * (m->QN + 2 * m->KN));
    if (!st) st = dalloc(m, &m->q, R * m->QN);
    if (!st) st = dalloc(m, &m->ygu, R * 2 * (size_t)m->F);
    if (!st) st = dalloc(m, &m->xn, R * m->hidden);
    if (!st && world == 1) st = dalloc(m, &m->logits, R * (size_t)m->V);
    if (!st) st = dalloc(m, &m->xi8, R * widest);
    if (!st) st = dalloc(m, &m->hq, R * (size_t)m->F);
    if (!st && R > 1)
        st = dalloc(m, &m->apart, (size_t)attn_part_floats((int)std::min<size_t>(R, 64), m->H, m->D, cfg->max_seq));
    m->lm_grid = lmhead_grid(ctx->device);
    if (!st) st = dalloc(m, &m->cand, (size_t)8 * m->lm_grid);
    if (!st) st = dalloc(m, &m->tok, (size_t)m->B);
    if (!st) st = dalloc(m, &m->tok_tmp, R);
    if (!st) st = dalloc(m, &m->ids, R);
    if (!st) st = dalloc(m, &m->row_seq, R);
    if (!st) st = dalloc(m, &m->row_i, R);
    if (!st) st = dalloc(m, &m->seqs, (size_t)m->B);
    if (!st) st = dalloc(m, &m->hist, (size_t)m->max_steps * m->B);
    if (!st) st = dalloc(m, &m->step_ctr, 1);
    if (!st) st = dalloc(m, &m->draws, (size_t)m->B);
    if (world == 1) {
        if (!st) st = dalloc(m, &m->cacc, R * m->hidden);
        if (!st) st = dalloc(m, &m->pairs, R);
        if (!st) st = dalloc(m, &m->pairs_all, R);
    } else {
        // buffers of collectives belong to the communicator (see q35_tp.cu)
        void *p = nullptr;
        if (!st) st = tp_buffer(tp, 0, sizeof(int32_t) * R * m->hidden, &p);
        m->cacc = static_cast<int32_t *>(p);
        if (!st) st = tp_buffer(tp, 1, sizeof(float2) * R, &p);
        m->pairs = static_cast<float2 *>(p);
        if (!st) st = tp_buffer(tp, 2, sizeof(float2) * R * world, &p);
        m->pairs_all = static_cast<float2 *>(p);
        if (!st) st = tp_buffer(tp, 3, sizeof(float) * R * (size_t)m->V, &p);
        m->logits = static_cast<float *>(p);
        if (!st) st = tp_buffer(tp, 4, sizeof(float) * R * (size_t)m->V * world, &p);
        m->logits_all = static_cast<float *>(p);
    }
    if (!st) st = dalloc(m, &m->embed, (size_t)m->Vg * m->hidden);
    if (!st) st = dalloc(m, &m->final_norm, (size_t)m->hidden);
    if (!st) st = dalloc(m, &m->lm_head, (size_t)m->V * m->hidden);
    for (int l = 0; l < m->L && !st; ++l) {
        st = dalloc(m, &m->layers[l].attn_norm, (size_t)m->hidden);
        if (!st) st = dalloc(m, &m->layers[l].ffn_norm, (size_t)m->hidden);
    }
    if (!st) {
        // norms start at 1.0 (llama_model.f90:74-75, transformer_layer.f90 init)
        const std::vector<float> ones((size_t)m->hidden, 1.0f);
        cudaError_t e = cudaSuccess;
        for (int l = 0; l < m->L && e == cudaSuccess; ++l) {
            e = cudaMemcpy(m->layers[l].attn_norm, ones.data(), sizeof(float) * m->hidden, cudaMemcpyHostToDevice);
            if (e == cudaSuccess)
                e = cudaMemcpy(m->layers[l].ffn_norm, ones.data(), sizeof(float) * m->hidden, cudaMemcpyHostToDevice);
        }
        if (e == cudaSuccess) e = cudaMemcpy(m->final_norm, ones.data(), sizeof(float) * m->hidden, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(m->rope, rt.data(), rt.size() * sizeof(float2), cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemset(m->kc, 0, kv * sizeof(float));
        if (e == cudaSuccess) e = cudaMemset(m->vc, 0, kv * sizeof(float));
        if (e == cudaSuccess) e = cudaMemset(m->cache_pos, 0, sizeof(int32_t) * m->B);
        if (e == cudaSuccess) e = cudaMemset(m->draws, 0, sizeof(int32_t) * m->B);
        // the decode graph reads the step counter and the previous tokens on its first replay
        if (e == cudaSuccess) e = cudaMemset(m->step_ctr, 0, sizeof(int32_t));
        if (e == cudaSuccess) e = cudaMemset(m->tok, 0, sizeof(int32_t) * m->B);
        if (e == cudaSuccess) e = cudaMemset(m->hist, 0, sizeof(int32_t) * (size_t)m->max_steps * m->B);
        if (e != cudaSuccess) st = set_error(Q35_ERR_CUDA, cudaGetErrorString(e));
    }
    m->host_pos.assign(m->B, 0);
    // workspace for every matmul the model issues (both engines, up to maxR rows),
    // sized before any capture
    if (!st) {
        Weights probe{};
        probe.format = cfg->wformat;
        probe.K = std::max({m->hidden, m->QN, m->F});
        probe.KB = (int32_t)ceil_div(probe.K, KBLK);
        probe.N = std::max({2 * m->F, m->QN + 2 * m->KN, m->hidden});
        probe.CG = (int32_t)ceil_div(probe.N, CGW);
        probe.device = ctx->device;
        probe.tile_bytes = cfg->wformat == Q35_FMT_3P5BIT ? TILE35 : TILE4;
        for (int32_t M : {1, (int32_t)m->B, 64, (int32_t)std::min<size_t>(R, 256), (int32_t)R})
            if (!st) st = ensure_gemm_workspace(ctx, probe, M);
    }
    if (st) {
        q35_model_destroy(m);
        return st;
    }
    *out = m;
    return Q35_OK;
}

int q35_model_destroy(q35_model m) {
    if (!m) return Q35_OK;
    DeviceGuard g(m->ctx->device);
    cudaStreamSynchronize(m->ctx->stream);
    if (m->gexec) cudaGraphExecDestroy(m->gexec);
    if (m->g) cudaGraphDestroy(m->g);
    for (LayerW &w : m->layers) {
        q35_weights_free(w.qkv);
        q35_weights_free(w.o);
        q35_weights_free(w.gu);
        q35_weights_free(w.d);
    }
    for (void *p : m->allocs) cudaFree(p);
    tp_attach(m->tp, -1);
    delete m;
    return Q35_OK;
}

// the shard of a reference-layout W_Q(K/2,N): columns [c0, c0+nc) (contiguous) ...
static void cols_of(const int8_t *wq, int K, int c0, int nc, std::vector<int8_t> &dst, size_t at) {
    std::memcpy(dst.data() + at, wq + (size_t)c0 * (K / 2), (size_t)nc * (K / 2));
}
// ... or rows [r0, r0+nr) (nr even) of every column: pairs [r0/2, (r0+nr)/2)
static void rows_of(const int8_t *wq, int K, int N, int r0, int nr, std::vector<int8_t> &dst) {
    dst.resize((size_t)N * (nr / 2));
    for (int j = 0; j < N; ++j)
        std::memcpy(dst.data() + (size_t)j * (nr / 2), wq + (size_t)j * (K / 2) + r0 / 2, (size_t)nr / 2);
}

int q35_model_set_layer(q35_model m, int32_t l, const q35_layer_weights *w) {
    if (!m || !w) return set_error(Q35_ERR_INVALID, "NULL argument");
    if (l < 0 || l >= m->L) return set_error(Q35_ERR_INVALID, "layer index out of range");
    const int fmt = m->cfg.wformat;
    const bool f35 = fmt == Q35_FMT_3P5BIT;
    if (!w->wq || !w->wk || !w->wv || !w->wo || !w->wg || !w->wu || !w->wd || !w->sq || !w->sk || !w->sv ||
        !w->so || !w->sg || !w->su || !w->sd)
        return set_error(Q35_ERR_INVALID, "layer weights: NULL pointer");
    if (f35 && (!w->oq || !w->ok || !w->ov || !w->oo || !w->og || !w->ou || !w->od))
        return set_error(Q35_ERR_INVALID, "layer weights: 3.5-bit offsets missing");
    DeviceGuard g(m->ctx->device);
    LayerW &L = m->layers[l];
    const int hid = m->hidden, QN = m->QN, KN = m->KN, F = m->F, r = m->rank;
    const int QNg = m->Hg * m->D, Fg = m->Fg;
    std::vector<int8_t> b;
    std::vector<float> sc, of;
    // q|k|v: this rank's query and KV heads (columns)
    b.resize((size_t)(QN + 2 * KN) * (hid / 2));
    cols_of(w->wq, hid, r * QN, QN, b, 0);
    cols_of(w->wk, hid, r * KN, KN, b, (size_t)QN * (hid / 2));
    cols_of(w->wv, hid, r * KN, KN, b, (size_t)(QN + KN) * (hid / 2));
    concat_f({w->sq + r * QN, w->sk + r * KN, w->sv + r * KN}, {QN, KN, KN}, sc);
    if (f35) concat_f({w->oq + r * QN, w->ok + r * KN, w->ov + r * KN}, {QN, KN, KN}, of);
    int st = upload_matrix(m, &L.qkv, fmt, b.data(), sc.data(), f35 ? of.data() : nullptr, QN + 2 * KN, hid);
    // o: rows of this rank's heads, full output columns (scales/offsets whole)
    if (!st) {
        rows_of(w->wo, QNg, hid, r * QN, QN, b);
        st = upload_matrix(m, &L.o, fmt, b.data(), w->so, w->oo, hid, QN);
    }
    // gate|up: this rank's FFN columns, interleaved (column 2i = gate i, 2i+1 = up i) so
    // that a SwiGLU pair sits in neighbouring lanes of the matmul's epilogue
    if (!st) {
        const size_t cb = hid / 2;
        b.resize((size_t)2 * F * cb);
        sc.resize((size_t)2 * F);
        of.resize(f35 ? (size_t)2 * F : 0);
        for (int i = 0; i < F; ++i) {
            std::memcpy(b.data() + (size_t)(2 * i) * cb, w->wg + (size_t)(r * F + i) * cb, cb);
            std::memcpy(b.data() + (size_t)(2 * i + 1) * cb, w->wu + (size_t)(r * F + i) * cb, cb);
            sc[2 * i] = w->sg[r * F + i];
            sc[2 * i + 1] = w->su[r * F + i];
            if (f35) {
                of[2 * i] = w->og[r * F + i];
                of[2 * i + 1] = w->ou[r * F + i];
            }
        }
        st = upload_matrix(m, &L.gu, fmt, b.data(), sc.data(), f35 ? of.data() : nullptr, 2 * F, hid);
    }
    // down: rows of this rank's FFN columns
    if (!st) {
        rows_of(w->wd, Fg, hid, r * F, F, b);
        st = upload_matrix(m, &L.d, fmt, b.data(), w->sd, w->od, hid, F);
    }
    // norms: NULL keeps the current ones (1.0 after creation, llama_model.f90:74-75)
    if (!st) {
        cudaError_t e = cudaSuccess;
        if (w->attn_norm) e = cudaMemcpy(L.attn_norm, w->attn_norm, sizeof(float) * hid, cudaMemcpyHostToDevice);
        if (e == cudaSuccess && w->ffn_norm)
            e = cudaMemcpy(L.ffn_norm, w->ffn_norm, sizeof(float) * hid, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) st = set_error(Q35_ERR_CUDA, cudaGetErrorString(e));
    }
    return st;
}

int q35_model_set_embeddings(q35_model m, const float *embed, const float *final_norm, const float *lm_head) {
    if (!m || !embed || !final_norm || !lm_head) return set_error(Q35_ERR_INVALID, "NULL argument");
    // embed arrives as the reference's E(vocab, hidden) column-major; stored row-major
    const int64_t Vg = m->Vg;
    std::vector<float> t((size_t)Vg * m->hidden);
    for (int64_t j = 0; j < m->hidden; ++j)
        for (int64_t v = 0; v < Vg; ++v) t[(size_t)v * m->hidden + j] = embed[v + (size_t)Vg * j];
    return model_set_embeddings_rm(m, t.data(), final_norm, lm_head);
}

// random-init matrix (K, N), generated and quantized whole on the device (so every TP
// size holds the same weights), then this rank's columns [c0, c0+nc) of up to three
// column ranges, or its rows [r0, r0+nr), are repacked
struct Slice { int c0, nc; };
static int random_shard(q35_model m, q35_weights *slot, int K, int N, uint64_t seed, uint64_t tid, double sigma,
                        const std::vector<Slice> &cols, int r0, int nr, bool interleave = false) {
    const int fmt = m->cfg.wformat;
    cudaStream_t s = m->ctx->stream;
    float *W = nullptr, *sc = nullptr, *of = nullptr, *sc2 = nullptr, *of2 = nullptr;
    int8_t *wq = nullptr, *wq2 = nullptr;
    const size_t n = (size_t)K * N;
    int Nl = 0;
    for (const Slice &c : cols) Nl += c.nc;
    const int Kl = cols.empty() ? nr : K;
    if (cols.empty()) Nl = N;
    int st = Q35_OK;
    cudaError_t e = cudaMallocAsync(&W, n * 4, s);
    if (e == cudaSuccess) e = cudaMallocAsync(&wq, n / 2, s);
    if (e == cudaSuccess) e = cudaMallocAsync(&sc, (size_t)N * 4, s);
    if (e == cudaSuccess) e = cudaMallocAsync(&of, (size_t)N * 4, s);
    if (e == cudaSuccess) e = cudaMallocAsync(&wq2, (size_t)Nl * (Kl / 2), s);
    if (e == cudaSuccess) e = cudaMallocAsync(&sc2, (size_t)Nl * 4, s);
    if (e == cudaSuccess) e = cudaMallocAsync(&of2, (size_t)Nl * 4, s);
    if (e != cudaSuccess) st = set_error(Q35_ERR_NOMEM, std::string("init_random: ") + cudaGetErrorString(e));
    if (!st) st = q35_gen_normal_dev(W, (int64_t)n, seed, tid, sigma, s);
    if (!st) st = q35_quantize_dev(fmt, W, wq, sc, of, K, N, s);
    if (!st) {
        if (cols.empty()) {   // rows: pairs [r0/2, (r0+nr)/2) of every column
            e = cudaMemcpy2DAsync(wq2, nr / 2, wq + r0 / 2, K / 2, nr / 2, N, cudaMemcpyDeviceToDevice, s);
            if (e == cudaSuccess) e = cudaMemcpyAsync(sc2, sc, (size_t)N * 4, cudaMemcpyDeviceToDevice, s);
            if (e == cudaSuccess) e = cudaMemcpyAsync(of2, of, (size_t)N * 4, cudaMemcpyDeviceToDevice, s);
        } else if (interleave) {   // two equal slices, column by column: c0[0]+i, c0[1]+i, ...
            const size_t cb = K / 2;
            for (int q = 0; q < 2 && e == cudaSuccess; ++q) {
                const Slice &c = cols[q];
                e = cudaMemcpy2DAsync(wq2 + q * cb, 2 * cb, wq + (size_t)c.c0 * cb, cb, cb, c.nc, cudaMemcpyDeviceToDevice, s);
                if (e == cudaSuccess)
                    e = cudaMemcpy2DAsync(sc2 + q, 8, sc + c.c0, 4, 4, c.nc, cudaMemcpyDeviceToDevice, s);
                if (e == cudaSuccess)
                    e = cudaMemcpy2DAsync(of2 + q, 8, of + c.c0, 4, 4, c.nc, cudaMemcpyDeviceToDevice, s);
            }
        } else {
            size_t at = 0;
            for (const Slice &c : cols) {
                if (e == cudaSuccess)
                    e = cudaMemcpyAsync(wq2 + at * (K / 2), wq + (size_t)c.c0 * (K / 2), (size_t)c.nc * (K / 2),
                                        cudaMemcpyDeviceToDevice, s);
                if (e == cudaSuccess) e = cudaMemcpyAsync(sc2 + at, sc + c.c0, (size_t)c.nc * 4, cudaMemcpyDeviceToDevice, s);
                if (e == cudaSuccess) e = cudaMemcpyAsync(of2 + at, of + c.c0, (size_t)c.nc * 4, cudaMemcpyDeviceToDevice, s);
                at += c.nc;
            }
        }
        if (e != cudaSuccess) st = set_error(Q35_ERR_CUDA, cudaGetErrorString(e));
    }
    if (*slot) { q35_weights_free(*slot); *slot = nullptr; }
    if (!st) st = weights_alloc(m->ctx, fmt, Nl, Kl, slot);
    if (!st) st = weights_fill(m->ctx, *slot, wq2, sc2, fmt == Q35_FMT_3P5BIT ? of2 : nullptr, 1);
    for (void *p : {(void *)W, (void *)wq, (void *)sc, (void *)of, (void *)wq2, (void *)sc2, (void *)of2})
        if (p) cudaFreeAsync(p, s);
    e = cudaStreamSynchronize(s);
    if (!st && e != cudaSuccess) st = set_error(Q35_ERR_CUDA, cudaGetErrorString(e));
    return st;
}

int q35_model_init_random(q35_model m, uint64_t seed, double sigma) {
    if (!m) return set_error(Q35_ERR_INVALID, "model is NULL");
    DeviceGuard g(m->ctx->device);
    int st = Q35_OK;
    cudaStream_t s = m->ctx->stream;
    const int r = m->rank, QN = m->QN, KN = m->KN, F = m->F;
    const int QNg = m->Hg * m->D, KNg = m->KVHg * m->D, Fg = m->Fg;
    for (int l = 0; l < m->L && !st; ++l) {
        LayerW &L = m->layers[l];
        const uint64_t t0 = 1000ull + 16ull * l;
        // q|k|v generated as one (hidden, QN+2KN) matrix, gate|up as one (hidden, 2F)
        st = random_shard(m, &L.qkv, m->hidden, QNg + 2 * KNg, seed, t0 + 0, sigma,
                          {{r * QN, QN}, {QNg + r * KN, KN}, {QNg + KNg + r * KN, KN}}, 0, 0);
        if (!st) st = random_shard(m, &L.o, QNg, m->hidden, seed, t0 + 1, sigma, {}, r * QN, QN);
        if (!st)   // gate|up interleaved by column, as q35_model_set_layer lays it out
            st = random_shard(m, &L.gu, m->hidden, 2 * Fg, seed, t0 + 2, sigma, {{r * F, F}, {Fg + r * F, F}}, 0, 0, true);
        if (!st) st = random_shard(m, &L.d, Fg, m->hidden, seed, t0 + 3, sigma, {}, r * F, F);
        if (!st) st = q35_gen_normal_dev(L.attn_norm, m->hidden, seed, t0 + 4, sigma, s);
        if (!st) st = q35_gen_normal_dev(L.ffn_norm, m->hidden, seed, t0 + 5, sigma, s);
    }
    if (!st) st = q35_gen_normal_dev(m->embed, (int64_t)m->Vg * m->hidden, seed, 1, sigma, s);
    if (!st) st = q35_gen_normal_dev(m->final_norm, m->hidden, seed, 2, sigma, s);
    if (!st) {   // the LM head: this rank's rows of the whole (vocab, hidden) draw
        float *full = nullptr;
        cudaError_t e = cudaMallocAsync(&full, sizeof(float) * (size_t)m->Vg * m->hidden, s);
        if (e != cudaSuccess) return set_error(Q35_ERR_NOMEM, cudaGetErrorString(e));
        st = q35_gen_normal_dev(full, (int64_t)m->Vg * m->hidden, seed, 3, sigma, s);
        if (!st) {
            e = cudaMemcpyAsync(m->lm_head, full + (size_t)r * m->V * m->hidden, sizeof(float) * (size_t)m->V * m->hidden,
                                cudaMemcpyDeviceToDevice, s);
            if (e != cudaSuccess) st = set_error(Q35_ERR_CUDA, cudaGetErrorString(e));
        }
        cudaFreeAsync(full, s);
    }
    if (!st) {
        cudaError_t e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) st = set_error(Q35_ERR_CUDA, cudaGetErrorString(e));
    }
    return st;
}

// the next-token rule; the decode graph is captured again on the next step (under tensor
// parallelism every rank makes the same call at the same point)
int q35_model_set_sampling(q35_model m, const q35_sampling *cfg) {
    if (!m || !cfg) return set_error(Q35_ERR_INVALID, "NULL argument");
    if (cfg->mode != Q35_SAMPLE_GREEDY) {
        int st = sample_check(cfg->mode, m->Vg);
        if (st) return st;
    }
    DeviceGuard g(m->ctx->device);
    std::lock_guard<std::mutex> lk(m->ctx->mu);
    cudaStream_t s = m->ctx->stream;
    Q35_CUDA_TRY(cudaStreamSynchronize(s));
    if (m->gexec) { cudaGraphExecDestroy(m->gexec); m->gexec = nullptr; }
    if (m->g) { cudaGraphDestroy(m->g); m->g = nullptr; }
    m->samp = *cfg;
    Q35_CUDA_TRY(cudaMemsetAsync(m->draws, 0, sizeof(int32_t) * m->B, s));
    Q35_CUDA_TRY(cudaStreamSynchronize(s));
    return Q35_OK;
}

int q35_model_reset(q35_model m) {
    if (!m) return set_error(Q35_ERR_INVALID, "model is NULL");
    DeviceGuard g(m->ctx->device);
    cudaStream_t s = m->ctx->stream;
    const size_t kv = (size_t)m->B * m->L * m->KVH * m->cfg.max_seq * m->D;
    Q35_CUDA_TRY(cudaMemsetAsync(m->kc, 0, kv * sizeof(float), s));
    Q35_CUDA_TRY(cudaMemsetAsync(m->vc, 0, kv * sizeof(float), s));
    Q35_CUDA_TRY(cudaMemsetAsync(m->cache_pos, 0, sizeof(int32_t) * m->B, s));
    Q35_CUDA_TRY(cudaMemsetAsync(m->step_ctr, 0, sizeof(int32_t), s));
    Q35_CUDA_TRY(cudaMemsetAsync(m->draws, 0, sizeof(int32_t) * m->B, s));
    Q35_CUDA_TRY(cudaStreamSynchronize(s));
    std::fill(m->host_pos.begin(), m->host_pos.end(), 0);
    return Q35_OK;
}

int q35_model_forward(q35_model m, int32_t seq, const int32_t *ids, int32_t S, float *logits) {
    int st = check_ready(m);
    if (st) return st;
    if (seq < 0 || seq >= m->B) return set_error(Q35_ERR_INVALID, "sequence index out of range");
    if (S < 1 || !ids) return set_error(Q35_ERR_INVALID, "forward: no tokens");
    if (m->host_pos[seq] + S > m->cfg.max_seq) return set_error(Q35_ERR_INVALID, "forward: KV cache full (max_seq)");
    DeviceGuard g(m->ctx->device);
    std::lock_guard<std::mutex> lk(m->ctx->mu);
    cudaStream_t s = m->ctx->stream;
    std::vector<int32_t> rs(S, seq), ri(S);
    for (int i = 0; i < S; ++i) ri[i] = i;
    Q35_CUDA_TRY(cudaMemcpyAsync(m->ids, ids, sizeof(int32_t) * S, cudaMemcpyHostToDevice, s));
    Q35_CUDA_TRY(cudaMemcpyAsync(m->row_seq, rs.data(), sizeof(int32_t) * S, cudaMemcpyHostToDevice, s));
    Q35_CUDA_TRY(cudaMemcpyAsync(m->row_i, ri.data(), sizeof(int32_t) * S, cudaMemcpyHostToDevice, s));
    Q35_CUDA_TRY(cudaMemcpyAsync(m->seqs, &seq, sizeof(int32_t), cudaMemcpyHostToDevice, s));
    const int lm0 = logits ? 0 : S - 1, lmn = logits ? S : 1;
    st = forward_rows(m, S, lm0, lmn, m->tok_tmp, 1, S, logits != nullptr, lmn - 1);
    if (st) return st;
    // next token of the last position goes to tok[seq] for the decode steps
    Q35_CUDA_TRY(cudaMemcpyAsync(m->tok + seq, m->tok_tmp + (lmn - 1), sizeof(int32_t), cudaMemcpyDeviceToDevice, s));
    if (logits) {
        st = logits_to_host(m, S, logits);   // device [S][V] row-major -> (S, vocab) column-major
        if (st) return st;
    }
    Q35_CUDA_TRY(cudaStreamSynchronize(s));
    m->host_pos[seq] += S;
    return q35_ctx_device_error(m->ctx);
}

int q35_model_last_tokens(q35_model m, int32_t *tokens) {
    if (!m || !tokens) return set_error(Q35_ERR_INVALID, "NULL argument");
    DeviceGuard g(m->ctx->device);
    Q35_CUDA_TRY(cudaMemcpyAsync(tokens, m->tok, sizeof(int32_t) * m->B, cudaMemcpyDeviceToHost, m->ctx->stream));
    Q35_CUDA_TRY(cudaStreamSynchronize(m->ctx->stream));
    return Q35_OK;
}

// decode step over all B sequences; ids (host, [B]) overrides the device tokens when set
static int decode_enqueue(q35_model m) {
    // rows r -> sequence r at position 0 of the call
    return forward_rows(m, m->B, 0, m->B, m->tok, m->B, 1, m->gather_logits, 0);
}

int q35_model_decode_step(q35_model m, const int32_t *ids, int32_t *next, float *logits) {
    int st = check_ready(m);
    if (st) return st;
    for (int b = 0; b < m->B; ++b)
        if (m->host_pos[b] + 1 > m->cfg.max_seq) return set_error(Q35_ERR_INVALID, "decode: KV cache full (max_seq)");
    DeviceGuard g(m->ctx->device);
    std::lock_guard<std::mutex> lk(m->ctx->mu);
    cudaStream_t s = m->ctx->stream;
    if (ids) Q35_CUDA_TRY(cudaMemcpyAsync(m->tok, ids, sizeof(int32_t) * m->B, cudaMemcpyHostToDevice, s));
    if (!m->gexec && logits && m->world > 1) m->gather_logits = true;
    if (!m->gexec) {
        Q35_CUDA_TRY(cudaStreamSynchronize(s));
        // the step reads its ids from tok (the previous step's next tokens)
        Q35_CUDA_TRY(cudaStreamBeginCapture(s, cudaStreamCaptureModeRelaxed));
        decode_rows_kernel<<<1, 256, 0, s>>>(m->tok, m->ids, m->row_seq, m->row_i, m->seqs, m->B);
        cudaError_t ce = cudaGetLastError();
        int cst = ce == cudaSuccess ? decode_enqueue(m) : set_error(Q35_ERR_CUDA, cudaGetErrorString(ce));
        if (!cst) {
            record_kernel<<<1, 256, 0, s>>>(m->tok, m->hist, m->step_ctr, m->B, m->max_steps);
            if (cudaGetLastError() != cudaSuccess) cst = set_error(Q35_ERR_CUDA, "record kernel launch");
        }
        cudaError_t e = cudaStreamEndCapture(s, &m->g);
        if (cst) { if (m->g) { cudaGraphDestroy(m->g); m->g = nullptr; } return cst; }
        if (e == cudaSuccess) e = cudaGraphInstantiate(&m->gexec, m->g, 0);
        if (e != cudaSuccess) return set_error(Q35_ERR_CUDA, std::string("decode graph: ") + cudaGetErrorString(e));
    }
    Q35_CUDA_TRY(cudaGraphLaunch(m->gexec, s));
    for (int b = 0; b < m->B; ++b) m->host_pos[b] += 1;
    if (next) Q35_CUDA_TRY(cudaMemcpyAsync(next, m->tok, sizeof(int32_t) * m->B, cudaMemcpyDeviceToHost, s));
    if (logits) {
        if (m->world > 1 && !m->gather_logits) return set_error(Q35_ERR_STATE, "decode: logits need a graph built with them");
        int lst = logits_to_host(m, m->B, logits);
        if (lst) return lst;
    }
    if (next || logits) Q35_CUDA_TRY(cudaStreamSynchronize(s));
    return Q35_OK;
}

// enqueue n decode steps (graph replays) without host synchronisation
int q35_model_decode_steps_async(q35_model m, int32_t n) {
    int st = check_ready(m);
    if (st) return st;
    if (n < 0) return set_error(Q35_ERR_INVALID, "negative step count");
    for (int b = 0; b < m->B; ++b)
        if (m->host_pos[b] + n > m->cfg.max_seq) return set_error(Q35_ERR_INVALID, "decode: KV cache full (max_seq)");
    if (!m->gexec) {   // builds the graph with one synchronous step
        if (n == 0) return Q35_OK;
        st = q35_model_decode_step(m, nullptr, nullptr, nullptr);
        if (st) return st;
        --n;
    }
    DeviceGuard g(m->ctx->device);
    for (int i = 0; i < n; ++i) Q35_CUDA_TRY(cudaGraphLaunch(m->gexec, m->ctx->stream));
    for (int b = 0; b < m->B; ++b) m->host_pos[b] += n;
    return Q35_OK;
}

// llama_generate.f90:76-123 with greedy sampling, for all B sequences at once:
// prompts [B][prompt_len] (1-based ids), out_tokens [B][n_steps]; n_out[b] = tokens kept
// (stop_at_eos: the sequence ends before its first token 2, as :101-104)
int q35_model_generate(q35_model m, const int32_t *prompts, int32_t prompt_len, int32_t n_steps,
                       int32_t stop_at_eos, int32_t *out_tokens, int32_t *n_out) {
    int st = check_ready(m);
    if (st) return st;
    if (!prompts || !out_tokens || prompt_len < 1 || n_steps < 1) return set_error(Q35_ERR_INVALID, "generate: bad arguments");
    st = q35_model_reset(m);
    if (st) return st;
    // :109-113 stops once the sequence would exceed MAX_SEQ_LEN
    const int steps = std::min(n_steps, m->cfg.max_seq - prompt_len);
    if (steps < 1) return set_error(Q35_ERR_INVALID, "generate: prompt fills the KV cache");
    for (int b = 0; b < m->B && !st; ++b) st = q35_model_forward(m, b, prompts + (size_t)b * prompt_len, prompt_len, nullptr);
    if (st) return st;
    DeviceGuard g(m->ctx->device);
    cudaStream_t s = m->ctx->stream;
    // step 1 token = greedy of the prompt's last position (already in tok)
    Q35_CUDA_TRY(cudaMemsetAsync(m->step_ctr, 0, sizeof(int32_t), s));
    record_kernel<<<1, 256, 0, s>>>(m->tok, m->hist, m->step_ctr, m->B, m->max_steps);
    Q35_CUDA_TRY(cudaGetLastError());
    st = q35_model_decode_steps_async(m, steps - 1);
    if (st) return st;
    std::vector<int32_t> h((size_t)steps * m->B);
    Q35_CUDA_TRY(cudaMemcpyAsync(h.data(), m->hist, h.size() * sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    Q35_CUDA_TRY(cudaStreamSynchronize(s));
    st = q35_ctx_device_error(m->ctx);
    if (st) return st;
    for (int b = 0; b < m->B; ++b) {
        int n = 0;
        for (int t = 0; t < steps; ++t) {
            const int32_t tk = h[(size_t)t * m->B + b];
            if (stop_at_eos && tk == 2) break;
            out_tokens[(size_t)b * n_steps + t] = tk;
            ++n;
        }
        if (n_out) n_out[b] = n;
    }
    return Q35_OK;
}

// one transformer layer on host activations x (S, hidden) column-major for sequence seq
// (apply_transformer_layer, transformer_layer.f90:527-565); advances the sequence's
// position by S when advance != 0
int q35_model_layer_forward(q35_model m, int32_t layer, int32_t seq, const float *x, int32_t S, float *out,
                            int32_t advance) {
    int st = check_ready(m);
    if (st) return st;
    if (layer < 0 || layer >= m->L || seq < 0 || seq >= m->B || S < 1 || !x || !out)
        return set_error(Q35_ERR_INVALID, "layer_forward: bad arguments");
    if (m->host_pos[seq] + S > m->cfg.max_seq) return set_error(Q35_ERR_INVALID, "layer_forward: KV cache full");
    DeviceGuard g(m->ctx->device);
    std::lock_guard<std::mutex> lk(m->ctx->mu);
    cudaStream_t s = m->ctx->stream;
    std::vector<float> t((size_t)S * m->hidden);
    for (int i = 0; i < S; ++i)
        for (int j = 0; j < m->hidden; ++j) t[(size_t)i * m->hidden + j] = x[i + (size_t)S * j];
    std::vector<int32_t> rs(S, seq), ri(S);
    for (int i = 0; i < S; ++i) ri[i] = i;
    Q35_CUDA_TRY(cudaMemcpyAsync(m->x, t.data(), t.size() * sizeof(float), cudaMemcpyHostToDevice, s));
    Q35_CUDA_TRY(cudaMemcpyAsync(m->row_seq, rs.data(), sizeof(int32_t) * S, cudaMemcpyHostToDevice, s));
    Q35_CUDA_TRY(cudaMemcpyAsync(m->row_i, ri.data(), sizeof(int32_t) * S, cudaMemcpyHostToDevice, s));
    Q35_CUDA_TRY(cudaMemcpyAsync(m->seqs, &seq, sizeof(int32_t), cudaMemcpyHostToDevice, s));
    m->rows_one_seq = true;
    st = layer_rows(m, layer, S);
    if (!st && advance) st = launch_advance(m->cache_pos, m->seqs, 1, S, s);
    if (st) return st;
    Q35_CUDA_TRY(cudaMemcpyAsync(t.data(), m->x, t.size() * sizeof(float), cudaMemcpyDeviceToHost, s));
    Q35_CUDA_TRY(cudaStreamSynchronize(s));
    for (int i = 0; i < S; ++i)
        for (int j = 0; j < m->hidden; ++j) out[i + (size_t)S * j] = t[(size_t)i * m->hidden + j];
    if (advance) m->host_pos[seq] += S;
    return q35_ctx_device_error(m->ctx);
}

int q35_model_debug_buffer(q35_model m, const char *name, void *host, size_t bytes) {
    if (!m || !name || !host) return set_error(Q35_ERR_INVALID, "NULL argument");
    const void *src = nullptr;
    size_t cap = 0;
    const size_t R = (size_t)m->maxR;
    const std::string n(name);
    if (n == "x") { src = m->x; cap = R * m->hidden * 4; }
    else if (n == "yqkv") { src = m->yqkv; cap = R * (m->QN + 2 * m->KN) * 4; }
    else if (n == "q") { src = m->q; cap = R * m->QN * 4; }
    else if (n == "ygu") { src = m->ygu; cap = R * 2 * (size_t)m->F * 4; }
    else if (n == "xi8") { src = m->xi8; cap = R * (size_t)std::max({m->hidden, m->QN, m->F}); }
    else if (n == "hq") { src = m->hq; cap = R * (size_t)m->F; }
    else if (n == "kc") { src = m->kc; cap = (size_t)m->B * m->L * m->KVH * m->cfg.max_seq * m->D * 4; }
    else if (n == "vc") { src = m->vc; cap = (size_t)m->B * m->L * m->KVH * m->cfg.max_seq * m->D * 4; }
    else return set_error(Q35_ERR_INVALID, "debug_buffer: unknown buffer " + n);
    if (bytes > cap) return set_error(Q35_ERR_INVALID, "debug_buffer: more bytes than the buffer holds");
    DeviceGuard g(m->ctx->device);
    Q35_CUDA_TRY(cudaStreamSynchronize(m->ctx->stream));
    Q35_CUDA_TRY(cudaMemcpy(host, src, bytes, cudaMemcpyDeviceToHost));
    return Q35_OK;
}

size_t q35_model_weight_bytes(q35_model m) {
    if (!m) return 0;
    size_t b = 0;
    for (const LayerW &w : m->layers)
        b += q35_weights_device_bytes(w.qkv) + q35_weights_device_bytes(w.o) + q35_weights_device_bytes(w.gu) +
             q35_weights_device_bytes(w.d) + 2 * sizeof(float) * (size_t)m->hidden;
    return b + sizeof(float) * ((size_t)(m->Vg + m->V) * m->hidden + m->hidden);
}

}  // extern "C"
