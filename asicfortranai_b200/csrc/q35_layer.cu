// q35_layer.cu -- the non-matmul kernels of the LLaMA layer and model
// (transformer_layer.f90, llama_model.f90, sampling.f90), fp32 like the reference.
//
// Rows: a forward processes R rows; row r belongs to sequence row_seq[r] at position
// row_i[r] within the call; its absolute position is cache_pos[seq] + row_i[r].
// Activations are row-major [R][width].  KV cache: [seq][layer][kv_head][max_seq][D].
#include <algorithm>
#include <cfloat>

#include "q35_expf.h"
#include "q35_layer.cuh"

namespace q35 {

// programmatic dependent launch: every kernel here is launched with the
// programmatic-stream-serialization attribute; it lets the next kernel start and waits
// for its predecessor's results before reading them
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
static int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    Q35_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...));
    return Q35_OK;
}

// A kernel's dynamic shared memory limit is an attribute of the kernel on one device: set
// it once per device (done: that kernel's flags, indexed by device ordinal).
template <typename... KArgs>
static int smem_limit_once(bool (&done)[64], void (*kern)(KArgs...), size_t bytes) {
    int dev = 0;
    Q35_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return set_error(Q35_ERR_INVALID, "device ordinal out of range");
    if (!done[dev]) {
        Q35_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
        done[dev] = true;
    }
    return Q35_OK;
}

// ---------------------------------------------------------------------------------------
__device__ __forceinline__ float block_sum(float v, float *red) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    v = (threadIdx.x < nw) ? red[threadIdx.x] : 0.0f;
    if (w == 0)
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) red[32] = v;
    __syncthreads();
    return red[32];
}

__device__ __forceinline__ float block_max(float v, float *red) {
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    v = (threadIdx.x < nw) ? red[threadIdx.x] : -FLT_MAX;
    if (w == 0)
        for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) red[32] = v;
    __syncthreads();
    return red[32];
}


// ---------------------------------------------------------------------------------------
// llama_model.f90:123-125: x(i,:) = E(id,:), ids 1-based.  E row-major [vocab][hidden]
// (hidden a multiple of 4): CTA (r, c) copies float4s [256 c, 256 c + 256) of row r, one per
// thread, so the row's loads are all in flight at once.
__global__ void embed_kernel(const int32_t *__restrict__ ids, const float *__restrict__ E,
                             float *__restrict__ x, int32_t hidden, int32_t vocab, int *err) {
    pdl_trigger();
    pdl_wait();
    const int r = blockIdx.x;
    const int id = ids[r];
    const bool ok = id >= 1 && id <= vocab;
    if (!ok && threadIdx.x == 0 && blockIdx.y == 0) atomicExch(err, Q35_ERR_INVALID);
    const int j = blockIdx.y * blockDim.x + threadIdx.x;
    if (j >= hidden / 4) return;
    const float4 *src = reinterpret_cast<const float4 *>(E + (size_t)(ok ? id - 1 : 0) * hidden);
    reinterpret_cast<float4 *>(x + (size_t)r * hidden)[j] = ok ? src[j] : make_float4(0.f, 0.f, 0.f, 0.f);
}

// transformer_layer.f90:155-178 rms_norm (+ the int8 quantization of int4_linear when
// q is non-null), float4 accesses (dim multiple of 4).  The row's sum of squares is the
// same in every launch shape: thread t of NORM_THREADS sums float4s t, t + NORM_THREADS, ...
// in order, then block_sum.  Elementwise part: with split == 1 one CTA per row writes the
// whole row; with split == 4 * ceil(dim / (4 * NORM_THREADS)) (few rows) CTA (r, p)
// recomputes the row's sum and writes component p % 4 of float4s t + (p / 4) * NORM_THREADS,
// so a thread divides one element instead of up to 4 * NORM_KMAX.  The weights do not depend
// on the previous kernel and are read before the dependency wait.
constexpr int NORM_THREADS = 1024;
constexpr int NORM_KMAX = 4;   // float4s per thread held in registers: dim <= 16384

__device__ __forceinline__ float f4_get(const float4 &v, int c) {
    return c == 0 ? v.x : (c == 1 ? v.y : (c == 2 ? v.z : v.w));
}

__device__ __forceinline__ void norm_store(const float4 v, const float4 g, float rms, float *__restrict__ out,
                                           int8_t *__restrict__ q, size_t base, int j) {
    const float4 o = make_float4(__fmul_rn(__fdiv_rn(v.x, rms), g.x), __fmul_rn(__fdiv_rn(v.y, rms), g.y),
                                 __fmul_rn(__fdiv_rn(v.z, rms), g.z), __fmul_rn(__fdiv_rn(v.w, rms), g.w));
    if (out) reinterpret_cast<float4 *>(out + base)[j] = o;
    if (q) {
        char4 c;
        c.x = quant127(o.x); c.y = quant127(o.y); c.z = quant127(o.z); c.w = quant127(o.w);
        reinterpret_cast<char4 *>(q + base)[j] = c;
    }
}

__global__ void __launch_bounds__(NORM_THREADS)
rmsnorm_kernel(const float *__restrict__ x, const float *__restrict__ w, float *__restrict__ out,
               int8_t *__restrict__ q, int32_t dim, float eps, int32_t split) {
    __shared__ float red[33];
    pdl_trigger();
    const int r = blockIdx.x, p = blockIdx.y, t = threadIdx.x;
    const int n4 = dim / 4, K4 = (n4 + NORM_THREADS - 1) / NORM_THREADS;
    const bool regs = K4 <= NORM_KMAX;
    const float4 *xr = reinterpret_cast<const float4 *>(x + (size_t)r * dim);
    const float4 *w4 = reinterpret_cast<const float4 *>(w);
    const int pk = p >> 2, pc = p & 3;                // split > 1: this CTA's float4 slot, component
    const int pj = t + pk * NORM_THREADS;
    float4 g[NORM_KMAX];
    float gs = 0.0f;
    if (regs) {
        if (split == 1) {
#pragma unroll
            for (int k = 0; k < NORM_KMAX; ++k) {
                const int j = t + k * NORM_THREADS;
                if (k < K4 && j < n4) g[k] = w4[j];
            }
        } else if (pj < n4) {
            gs = w[4 * pj + pc];
        }
    }
    pdl_wait();
    float4 v[NORM_KMAX];
    float s = 0.0f;
    if (regs) {
#pragma unroll
        for (int k = 0; k < NORM_KMAX; ++k) {
            const int j = t + k * NORM_THREADS;
            if (k < K4 && j < n4) {
                v[k] = xr[j];
                s = __fadd_rn(s, __fmul_rn(v[k].x, v[k].x));
                s = __fadd_rn(s, __fmul_rn(v[k].y, v[k].y));
                s = __fadd_rn(s, __fmul_rn(v[k].z, v[k].z));
                s = __fadd_rn(s, __fmul_rn(v[k].w, v[k].w));
            }
        }
    } else {
        for (int j = t; j < n4; j += NORM_THREADS) {
            const float4 u = xr[j];
            s = __fadd_rn(s, __fmul_rn(u.x, u.x));
            s = __fadd_rn(s, __fmul_rn(u.y, u.y));
            s = __fadd_rn(s, __fmul_rn(u.z, u.z));
            s = __fadd_rn(s, __fmul_rn(u.w, u.w));
        }
    }
    s = block_sum(s, red);
    const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)dim), eps));
    if (regs && split > 1) {
        if (pj < n4) {
            float4 u = v[0];
#pragma unroll
            for (int k = 1; k < NORM_KMAX; ++k)
                if (k == pk) u = v[k];
            const float o = __fmul_rn(__fdiv_rn(f4_get(u, pc), rms), gs);
            const size_t oi = (size_t)r * dim + 4 * pj + pc;
            if (out) out[oi] = o;
            if (q) q[oi] = quant127(o);
        }
        return;
    }
#pragma unroll
    for (int k = 0; k < NORM_KMAX; ++k) {
        if (!regs) break;
        const int j = t + k * NORM_THREADS;
        if (k >= K4 || j >= n4) continue;
        norm_store(v[k], g[k], rms, out, q, (size_t)r * dim, j);
    }
    if (!regs)
        for (int j = t; j < n4; j += NORM_THREADS) norm_store(xr[j], w4[j], rms, out, q, (size_t)r * dim, j);
}

// transformer_layer.f90:183-205 (RoPE on q and k, interleaved pairs (2d, 2d+1)) and
// :322-329 (K/V written to the cache at cache_pos + i).  Input: the fused q|k|v output
// [R][QN + 2KN].  The rotation angle's position is the row's index within the call
// (rope_mode 0, the reference's apply_rope_single, :193-196) or its absolute position
// (rope_mode 1).  cs: [max_seq][D/2] pairs (cos, sin) computed on the host.
__global__ void rope_kv_kernel(const float *__restrict__ yqkv, float *__restrict__ q,
                               float *__restrict__ kc, float *__restrict__ vc,
                               const int32_t *__restrict__ row_seq, const int32_t *__restrict__ row_i,
                               const int32_t *__restrict__ cache_pos, const float2 *__restrict__ cs,
                               int32_t layer, int32_t n_layers, int32_t H, int32_t KVH, int32_t D,
                               int32_t max_seq, int32_t rope_mode, int *err) {
    // grid: (row, head) with heads 0..H-1 the queries, H..H+KVH-1 the keys (+ values)
    pdl_trigger();
    pdl_wait();
    const int r = blockIdx.x, hh = blockIdx.y;
    const int s = row_seq[r], i = row_i[r];
    const int pos = cache_pos[s] + i;
    if (pos < 0 || pos >= max_seq) {
        if (threadIdx.x == 0 && hh == 0) atomicExch(err, Q35_ERR_INVALID);
        return;
    }
    const int rp = rope_mode ? pos : i;
    const int QN = H * D, KN = KVH * D, W = QN + 2 * KN;
    const float *y = yqkv + (size_t)r * W;
    const int half = D / 2;
    const bool isq = hh < H;
    const int kh = hh - H;
    const int col0 = isq ? hh * D : QN + kh * D;
    for (int d = threadIdx.x; d < half; d += blockDim.x) {
        const float2 c = cs[(size_t)rp * half + d];
        const float2 ab = *reinterpret_cast<const float2 *>(y + col0 + 2 * d);
        const float ra = __fsub_rn(__fmul_rn(ab.x, c.x), __fmul_rn(ab.y, c.y));
        const float rb = __fadd_rn(__fmul_rn(ab.x, c.y), __fmul_rn(ab.y, c.x));
        if (isq) {
            *reinterpret_cast<float2 *>(q + (size_t)r * QN + hh * D + 2 * d) = make_float2(ra, rb);
        } else {
            const size_t o = ((((size_t)s * n_layers + layer) * KVH + kh) * max_seq + pos) * D + 2 * d;
            *reinterpret_cast<float2 *>(kc + o) = make_float2(ra, rb);
            *reinterpret_cast<float2 *>(vc + o) = *reinterpret_cast<const float2 *>(y + QN + KN + kh * D + 2 * d);
        }
    }
}

// Every fp32 reduction below runs in a fixed order (per-thread fused chains, 32-lane xor
// butterflies, chunk merges in chunk order) and every exponential is q35_expf, so the
// results are reproducible bit for bit by a CPU restatement of the same order.
//
// transformer_layer.f90:333-402 over chunks of ATT_CHUNK keys (flash-decoding), one
// thread-block cluster of cs = min(8, chunks of the cache) CTAs per (row, KV head group):
// the group's query heads (kv_h = (h-1)/(H/KVH)+1, :342) share each key and value.  CTA k
// of the cluster takes chunks k, k+cs, k+2cs, ...: their keys and values (contiguous in the
// cache) arrive by bulk copies into a shared-memory stage (double-buffered when a CTA has
// more than one chunk), and per chunk and head the CTA keeps, in
// its own shared memory, the chunk's max score m, sum l of exp(s - m) and o = sum
// exp(s-m) v.  After a cluster barrier CTA k merges head k of the group: it reads every
// chunk's (m, l, o) through distributed shared memory and combines them in chunk order
// (exp(m_c - M) rescaling), normalises and quantizes to int8 for the o-projection -- no
// global round trip.  Keys j > pos are the reference's masked entries (score -1e9,
// weight exp(-1e9 - max) = 0) and are skipped, chunks past pos entirely.
constexpr int ATT_CHUNK = 64;
constexpr int ATT_MAXG = 8;       // query heads per KV head handled by one cluster
constexpr int ATT_CS = 8;         // CTAs per cluster, at most
constexpr int ATT_MAX_CHUNKS = 128;   // max_seq <= 8192
constexpr int ATT1_THREADS = 256;     // the one-row kernel (attn_kernel)
constexpr int ATT_PSTR = 33;          // padded row of the 32 lane partials of one (key, head)

__device__ __forceinline__ bool att_wait(uint32_t bar, uint32_t parity) {
    for (uint32_t i = 0; i < (1u << 24); ++i) {
        uint32_t ok;
        asm volatile("{\n\t.reg .pred P1;\n\t"
                     "mbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2;\n\t"
                     "selp.b32 %0, 1, 0, P1;\n\t}"
                     : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
        if (ok) return true;
    }
    return false;
}
__device__ __forceinline__ uint32_t cta_rank_in_cluster() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// generic address of the same shared-memory variable in CTA `rank` of the cluster
// store v into the same shared-memory location of CTA `rank` of the cluster
__device__ __forceinline__ void st_cluster_f32(float *local, uint32_t rank, float v) {
    uint32_t ra;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
                 : "=r"(ra) : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(local))), "r"(rank));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(ra), "f"(v) : "memory");
}
template <typename T>
__device__ __forceinline__ const T *peer_smem(const T *p, uint32_t rank) {
    uint64_t out;
    asm volatile("mapa.u64 %0, %1, %2;" : "=l"(out) : "l"(reinterpret_cast<uint64_t>(p)), "r"(rank));
    return reinterpret_cast<const T *>(out);
}

// FLEX: cluster size, stage buffers and the score-partial stride from the launch (short
// contexts, narrow groups); otherwise the full shape as compile-time constants (8-CTA
// clusters, double-buffered stages at head_dim 128, partials of ATT_MAXG heads)
template <int D4, bool FLEX>   // head_dim / 128
__global__ void __launch_bounds__(ATT1_THREADS)
attn_kernel(const float *__restrict__ q, const float *__restrict__ kc, const float *__restrict__ vc,
            int8_t *__restrict__ out_q, float *__restrict__ out_f, const int32_t *__restrict__ row_seq,
            const int32_t *__restrict__ row_i, const int32_t *__restrict__ cache_pos, int32_t layer,
            int32_t n_layers, int32_t H, int32_t KVH, int32_t max_seq, int32_t mbf, int32_t nb_arg,
            int32_t cs_arg, int32_t use_part, int *err) {
    constexpr int D = 128 * D4;
    // dynamic: K,V stage x nb (2: the next chunk of this CTA streams in during the current
    // one; 1 when a CTA has one chunk at most, or at head_dim 256) | merge buffer: the
    // (o, m, l) partials of every chunk for the heads this CTA merges, [MH][nchunk][D + 2]
    // (mbf floats, written by the cluster's CTAs) | 2 mbarriers | (use_part: head_dim 128
    // where it fits) lane partials of the scores [ATT_CHUNK][gp][ATT_PSTR], gp = the group's
    // heads (<= ATT_MAXG)
    // [ATT_CHUNK][ATT_MAXG][ATT_PSTR]
    extern __shared__ __align__(128) float att_smem[];
    __shared__ float sc[ATT_MAXG][ATT_CHUNK];
    __shared__ float red[ATT_MAXG][2];
    __shared__ float cm[ATT_MAX_CHUNKS], cw[ATT_MAX_CHUNKS];
    __shared__ float cML[2];
    pdl_trigger();
    const uint32_t crank = cta_rank_in_cluster();
    const int cs = FLEX ? cs_arg : ATT_CS;
    const int nb = FLEX ? nb_arg : (D4 == 1 ? 2 : 1);
    const int r = blockIdx.x, grp = blockIdx.y / cs;
    const int kvh = grp % KVH, gpart = grp / KVH;
    const int G = H / KVH;
    const int g0 = gpart * ATT_MAXG, ng = min(ATT_MAXG, G - g0);
    const int gp = FLEX ? min(G, ATT_MAXG) : ATT_MAXG;
    const int nchunk = (max_seq + ATT_CHUNK - 1) / ATT_CHUNK;
    float *stage = att_smem;                                   // [nb][2][ATT_CHUNK][D]
    float *mb = att_smem + (size_t)nb * 2 * ATT_CHUNK * D;     // [MH][nchunk][D + 2]
    const uint32_t bar0 = static_cast<uint32_t>(__cvta_generic_to_shared(mb + mbf));
    float *part = mb + mbf + 4;   // after the two mbarriers (16 B)
    if (threadIdx.x == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar0) : "memory");
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar0 + 8) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    pdl_wait();
    const int s = row_seq[r];
    const int pos = cache_pos[s] + row_i[r];
    const int QN = H * D;
    const int n_act = (pos < 0 || pos >= max_seq) ? 0 : pos / ATT_CHUNK + 1;   // chunks holding keys <= pos
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t base = (((size_t)s * n_layers + layer) * KVH + kvh) * max_seq * D;
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)D));   // :336
    auto issue = [&](int c, int b) {   // chunk c into stage buffer b
        const int nj = min(ATT_CHUNK, pos + 1 - c * ATT_CHUNK);
        const uint32_t bytes = (uint32_t)(nj * D * 4);
        const uint32_t bar = bar0 + 8u * b;
        float *Ks = stage + (size_t)b * 2 * ATT_CHUNK * D, *Vs = Ks + (size_t)ATT_CHUNK * D;
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(2 * bytes) : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                     ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(Ks))), "l"(kc + base + (size_t)c * ATT_CHUNK * D),
                       "r"(bytes), "r"(bar) : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                     ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(Vs))), "l"(vc + base + (size_t)c * ATT_CHUNK * D),
                       "r"(bytes), "r"(bar) : "memory");
    };
    __syncthreads();   // barriers initialised
    if (threadIdx.x == 0 && (int)crank < n_act) issue(crank, 0);
    // q of the group in registers: lane holds dims [4*lane + 128*t, +4)
    float4 qv[ATT_MAXG][D4];
#pragma unroll
    for (int g = 0; g < ATT_MAXG; ++g)
#pragma unroll
        for (int t = 0; t < D4; ++t)
            qv[g][t] = (g < ng) ? *reinterpret_cast<const float4 *>(q + (size_t)r * QN + (kvh * G + g0 + g) * D + 128 * t + 4 * lane)
                                : make_float4(0, 0, 0, 0);
    int it = 0;
    for (int c = crank; c < n_act; c += cs, ++it) {
        const int b = nb == 2 ? (it & 1) : 0;
        const uint32_t par = nb == 2 ? (uint32_t)((it >> 1) & 1) : (uint32_t)(it & 1);
        // with two buffers the next chunk of this CTA streams in while this one is computed
        if (nb == 2 && threadIdx.x == 0 && c + cs < n_act) issue(c + cs, b ^ 1);
        if (!att_wait(bar0 + 8u * b, par)) {
            atomicExch(err, Q35_ERR_TIMEOUT);
            att_wait(bar0 + 8u * b, par);   // bounded
        }
        const float *Ks = stage + (size_t)b * 2 * ATT_CHUNK * D, *Vs = Ks + (size_t)ATT_CHUNK * D;
        const int nj = min(ATT_CHUNK, pos + 1 - c * ATT_CHUNK);
        for (int j = warp; j < nj; j += ATT1_THREADS / 32) {
            float a[ATT_MAXG];
#pragma unroll
            for (int g = 0; g < ATT_MAXG; ++g) a[g] = 0.0f;
#pragma unroll
            for (int t = 0; t < D4; ++t) {
                const float4 k4 = *reinterpret_cast<const float4 *>(Ks + (size_t)j * D + 128 * t + 4 * lane);
#pragma unroll
                for (int g = 0; g < ATT_MAXG; ++g)
                    a[g] = fmaf(qv[g][t].x, k4.x, fmaf(qv[g][t].y, k4.y, fmaf(qv[g][t].z, k4.z, fmaf(qv[g][t].w, k4.w, a[g]))));
            }
            if (D4 == 1 && use_part) {
                // the lanes' partials to shared memory; their sum below takes the butterfly's
                // pairing, so the score is the one the xor butterfly gives
                float *pp = part + (size_t)j * gp * ATT_PSTR + lane;
#pragma unroll
                for (int g = 0; g < ATT_MAXG; ++g)
                    if (g < gp) pp[g * ATT_PSTR] = a[g];
            } else {
#pragma unroll
                for (int g = 0; g < ATT_MAXG; ++g) {
                    float v = a[g];
                    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                    if (lane == 0 && g < ng) sc[g][j] = __fmul_rn(v, scale);
                }
            }
        }
        __syncthreads();
        if (D4 == 1 && use_part) {
            // one thread per (key, head): the 32 lane partials added in the xor butterfly's
            // pairing (step o adds partial l + o to partial l, o = 16, 8, 4, 2, 1: lane 0's
            // value; every lane of the butterfly ends with it, addition being commutative)
            for (int pr = threadIdx.x; pr < nj * gp; pr += ATT1_THREADS) {
                const int j = pr / gp, g = pr % gp;
                if (g >= ng) continue;
                const float *pp = part + (size_t)pr * ATT_PSTR;
                float w[32];
#pragma unroll
                for (int l = 0; l < 32; ++l) w[l] = pp[l];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                    for (int l = 0; l < o; ++l) w[l] = w[l] + w[l + o];
                sc[g][j] = __fmul_rn(w[0], scale);
            }
            __syncthreads();
        }
        // per head: chunk max and exp sums (warp g handles head g)
        for (int g = warp; g < ng; g += ATT1_THREADS / 32) {
            float m = -INFINITY;
            for (int j = lane; j < nj; j += 32) m = fmaxf(m, sc[g][j]);
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            float l = 0.0f;
            for (int j = lane; j < nj; j += 32) {
                const float e = q35_expf(__fsub_rn(sc[g][j], m));
                sc[g][j] = e;
                l += e;
            }
            for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
            if (lane == 0) { red[g][0] = m; red[g][1] = l; }
        }
        __syncthreads();
        // o[g][d] = sum_j e[g][j] * v[j][d] (in j order); thread t takes dimension t % D and
        // the heads of group t / D.  Head g's partials go straight into the merge buffer of
        // CTA g % cs (distributed shared-memory stores, ordered by the cluster barrier below)
        {
            constexpr int HQ = ATT1_THREADS / D, HPT = ATT_MAXG / HQ;
            const int d = threadIdx.x % D, gq = threadIdx.x / D;
            float o[HPT];
#pragma unroll
            for (int h = 0; h < HPT; ++h) o[h] = 0.0f;
            for (int j = 0; j < nj; ++j) {
                const float v = Vs[(size_t)j * D + d];
#pragma unroll
                for (int h = 0; h < HPT; ++h) o[h] = fmaf(sc[gq * HPT + h][j], v, o[h]);
            }
#pragma unroll
            for (int h = 0; h < HPT; ++h) {
                const int g = gq * HPT + h;
                if (g < ng) st_cluster_f32(mb + ((size_t)(g / cs) * nchunk + c) * (D + 2) + d, (uint32_t)(g % cs), o[h]);
            }
        }
        if (threadIdx.x < ng) {
            const int g = threadIdx.x;
            float *dst = mb + ((size_t)(g / cs) * nchunk + c) * (D + 2) + D;
            st_cluster_f32(dst, (uint32_t)(g % cs), red[g][0]);
            st_cluster_f32(dst + 1, (uint32_t)(g % cs), red[g][1]);
        }
        __syncthreads();   // sc and this stage buffer are reused
        if (nb == 1 && threadIdx.x == 0 && c + cs < n_act) issue(c + cs, 0);
    }
    cluster_sync_all();   // every chunk's partial is in its merging CTA's shared memory
    // merge: CTA k of the cluster merges heads k, k + cs, ... from its own merge buffer
    for (int g = (int)crank; g < ng; g += cs) {
        const float *hb = mb + (size_t)(g / cs) * nchunk * (D + 2);
        for (int c = threadIdx.x; c < n_act; c += blockDim.x) {
            cm[c] = hb[(size_t)c * (D + 2) + D];
            cw[c] = hb[(size_t)c * (D + 2) + D + 1];   // l for now
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            float M = -INFINITY;
            for (int c = 0; c < n_act; ++c) M = fmaxf(M, cm[c]);
            float L = 0.0f;
            for (int c = 0; c < n_act; ++c) L = fmaf(cw[c], q35_expf(__fsub_rn(cm[c], M)), L);
            cML[0] = M;
            cML[1] = L;
        }
        __syncthreads();
        for (int c = threadIdx.x; c < n_act; c += blockDim.x) cw[c] = q35_expf(__fsub_rn(cm[c], cML[0]));
        __syncthreads();
        const int h = kvh * G + g0 + g;
        for (int d = threadIdx.x; d < D; d += ATT1_THREADS) {
            float a = 0.0f;
#pragma unroll 4
            for (int c = 0; c < n_act; ++c) a = fmaf(hb[(size_t)c * (D + 2) + d], cw[c], a);
            const float v = __fdiv_rn(a, cML[1]);
            const size_t oi = (size_t)r * H * D + (size_t)h * D + d;
            if (out_q) out_q[oi] = quant127(v);
            if (out_f) out_f[oi] = v;
        }
        __syncthreads();
    }
    // no distributed shared-memory access follows the barrier above: CTAs exit on their own
}

// Many rows (decode batches, prefill): enough parallelism without clusters.  One CTA per
// (row, KV head group, chunk) computes the chunk partials exactly as above -- the chunk's
// keys and values arrive in shared memory by two bulk copies (reading them from global
// memory key by key left each CTA waiting on one load latency per key) -- into a global
// buffer; attn_combine_kernel, one CTA per (row, head), merges them in chunk order.
template <int D4>
__global__ void __launch_bounds__(ATT1_THREADS)
attn_partial_kernel(const float *__restrict__ q, const float *__restrict__ kc, const float *__restrict__ vc,
                    float *__restrict__ part, const int32_t *__restrict__ row_seq,
                    const int32_t *__restrict__ row_i, const int32_t *__restrict__ cache_pos, int32_t layer,
                    int32_t n_layers, int32_t H, int32_t KVH, int32_t max_seq, int32_t nchunk, int *err) {
    constexpr int D = 128 * D4;
    // dynamic: the chunk's keys and values [2][ATT_CHUNK][D], brought in by two bulk copies
    // (the keys of a chunk are contiguous in the cache), then their mbarrier
    extern __shared__ __align__(128) float att_smem[];
    __shared__ float sc[ATT_MAXG][ATT_CHUNK];
    __shared__ float red[ATT_MAXG][2];
    pdl_trigger();
    float *Ks = att_smem, *Vs = att_smem + (size_t)ATT_CHUNK * D;
    const uint32_t bar = static_cast<uint32_t>(__cvta_generic_to_shared(att_smem + (size_t)2 * ATT_CHUNK * D));
    pdl_wait();
    const int r = blockIdx.x, kvh = blockIdx.y % KVH, gpart = blockIdx.y / KVH, c = blockIdx.z;
    const int G = H / KVH;
    const int g0 = gpart * ATT_MAXG, ng = min(ATT_MAXG, G - g0);
    const int s = row_seq[r];
    const int pos = cache_pos[s] + row_i[r];
    const int QN = H * D;
    const int j0 = c * ATT_CHUNK;
    const int nj = (pos < 0 || pos >= max_seq) ? 0 : max(0, min(ATT_CHUNK, pos + 1 - j0));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // partial layout: [row][head][chunk][D + 2] -> o[D], m, l
    auto pout = [&](int h) { return part + (((size_t)r * H + h) * nchunk + c) * (D + 2); };
    if (nj == 0) {
        for (int g = 0; g < ng; ++g)
            if (threadIdx.x == 0) { pout(kvh * G + g0 + g)[D] = -INFINITY; pout(kvh * G + g0 + g)[D + 1] = 0.0f; }
        return;
    }
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)D));   // :336
    const size_t base = (((size_t)s * n_layers + layer) * KVH + kvh) * max_seq * D;
    if (threadIdx.x == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        const uint32_t bytes = (uint32_t)(nj * D * 4);
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(2 * bytes) : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                     ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(Ks))), "l"(kc + base + (size_t)j0 * D),
                       "r"(bytes), "r"(bar) : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                     ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(Vs))), "l"(vc + base + (size_t)j0 * D),
                       "r"(bytes), "r"(bar) : "memory");
    }
    // q of the group in registers while the copies land: lane holds dims [4*lane + 128*t, +4)
    float4 qv[ATT_MAXG][D4];
#pragma unroll
    for (int g = 0; g < ATT_MAXG; ++g)
#pragma unroll
        for (int t = 0; t < D4; ++t)
            qv[g][t] = (g < ng) ? *reinterpret_cast<const float4 *>(q + (size_t)r * QN + (kvh * G + g0 + g) * D + 128 * t + 4 * lane)
                                : make_float4(0, 0, 0, 0);
    __syncthreads();   // the barrier is initialised before anyone waits on it
    if (!att_wait(bar, 0)) {
        atomicExch(err, Q35_ERR_TIMEOUT);
        att_wait(bar, 0);   // bounded
    }
    for (int j = warp; j < nj; j += ATT1_THREADS / 32) {
        float a[ATT_MAXG];
#pragma unroll
        for (int g = 0; g < ATT_MAXG; ++g) a[g] = 0.0f;
#pragma unroll
        for (int t = 0; t < D4; ++t) {
            const float4 k4 = *reinterpret_cast<const float4 *>(Ks + (size_t)j * D + 128 * t + 4 * lane);
#pragma unroll
            for (int g = 0; g < ATT_MAXG; ++g)
                a[g] = fmaf(qv[g][t].x, k4.x, fmaf(qv[g][t].y, k4.y, fmaf(qv[g][t].z, k4.z, fmaf(qv[g][t].w, k4.w, a[g]))));
        }
#pragma unroll
        for (int g = 0; g < ATT_MAXG; ++g) {
            float v = a[g];
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0 && g < ng) sc[g][j] = __fmul_rn(v, scale);
        }
    }
    __syncthreads();
    // per head: chunk max and exp sums (warp g handles head g)
    for (int g = warp; g < ng; g += ATT1_THREADS / 32) {
        float m = -INFINITY;
        for (int j = lane; j < nj; j += 32) m = fmaxf(m, sc[g][j]);
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float l = 0.0f;
        for (int j = lane; j < nj; j += 32) {
            const float e = q35_expf(__fsub_rn(sc[g][j], m));
            sc[g][j] = e;
            l += e;
        }
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        if (lane == 0) { red[g][0] = m; red[g][1] = l; }
    }
    __syncthreads();
    // o[g][d] = sum_j e[g][j] * v[j][d] (in j order); thread t takes dimension t % D and the
    // heads of group t / D
    {
        constexpr int HQ = ATT1_THREADS / D, HPT = ATT_MAXG / HQ;
        const int d = threadIdx.x % D, gq = threadIdx.x / D;
        float o[HPT];
#pragma unroll
        for (int h = 0; h < HPT; ++h) o[h] = 0.0f;
        for (int j = 0; j < nj; ++j) {
            const float v = Vs[(size_t)j * D + d];
#pragma unroll
            for (int h = 0; h < HPT; ++h) o[h] = fmaf(sc[gq * HPT + h][j], v, o[h]);
        }
#pragma unroll
        for (int h = 0; h < HPT; ++h)
            if (gq * HPT + h < ng) pout(kvh * G + g0 + gq * HPT + h)[d] = o[h];
    }
    if (threadIdx.x < ng) {
        pout(kvh * G + g0 + threadIdx.x)[D] = red[threadIdx.x][0];
        pout(kvh * G + g0 + threadIdx.x)[D + 1] = red[threadIdx.x][1];
    }
}

// The same partials for rows that share one sequence (prefill): each CTA reads its chunk
// from global memory key by key; the rows of a sequence read the same chunks, which the
// SM's L1 then serves (bulk copies into each CTA's shared memory measured slower there).
constexpr int ATT_GLOBAL_THREADS = 128;
template <int D4>
__global__ void __launch_bounds__(ATT_GLOBAL_THREADS)
attn_partial_global_kernel(const float *__restrict__ q, const float *__restrict__ kc, const float *__restrict__ vc,
                    float *__restrict__ part, const int32_t *__restrict__ row_seq,
                    const int32_t *__restrict__ row_i, const int32_t *__restrict__ cache_pos, int32_t layer,
                    int32_t n_layers, int32_t H, int32_t KVH, int32_t D, int32_t max_seq, int32_t nchunk) {
    __shared__ float sc[ATT_MAXG][ATT_CHUNK];
    __shared__ float red[ATT_MAXG][2];
    pdl_trigger();
    pdl_wait();
    const int r = blockIdx.x, kvh = blockIdx.y % KVH, gpart = blockIdx.y / KVH, c = blockIdx.z;
    const int G = H / KVH;
    const int g0 = gpart * ATT_MAXG, ng = min(ATT_MAXG, G - g0);
    const int s = row_seq[r];
    const int pos = cache_pos[s] + row_i[r];
    const int QN = H * D;
    const int j0 = c * ATT_CHUNK;
    const int nj = (pos < 0 || pos >= max_seq) ? 0 : max(0, min(ATT_CHUNK, pos + 1 - j0));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // partial layout: [row][head][chunk][D + 2] -> o[D], m, l
    auto pout = [&](int h) { return part + (((size_t)r * H + h) * nchunk + c) * (D + 2); };
    if (nj == 0) {
        for (int g = 0; g < ng; ++g)
            if (threadIdx.x == 0) { pout(kvh * G + g0 + g)[D] = -INFINITY; pout(kvh * G + g0 + g)[D + 1] = 0.0f; }
        return;
    }
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)D));   // :336
    const size_t base = (((size_t)s * n_layers + layer) * KVH + kvh) * max_seq * D;
    const float *K = kc + base + (size_t)j0 * D, *V = vc + base + (size_t)j0 * D;
    // q of the group in registers: lane holds dims [4*lane + 128*t, +4)
    float4 qv[ATT_MAXG][D4];
#pragma unroll
    for (int g = 0; g < ATT_MAXG; ++g)
#pragma unroll
        for (int t = 0; t < D4; ++t)
            qv[g][t] = (g < ng) ? *reinterpret_cast<const float4 *>(q + (size_t)r * QN + (kvh * G + g0 + g) * D + 128 * t + 4 * lane)
                                          : make_float4(0, 0, 0, 0);
    for (int j = warp; j < nj; j += ATT_GLOBAL_THREADS / 32) {
        float a[ATT_MAXG];
#pragma unroll
        for (int g = 0; g < ATT_MAXG; ++g) a[g] = 0.0f;
#pragma unroll
        for (int t = 0; t < D4; ++t) {
            const float4 k4 = *reinterpret_cast<const float4 *>(K + (size_t)j * D + 128 * t + 4 * lane);
#pragma unroll
            for (int g = 0; g < ATT_MAXG; ++g)
                a[g] = fmaf(qv[g][t].x, k4.x, fmaf(qv[g][t].y, k4.y, fmaf(qv[g][t].z, k4.z, fmaf(qv[g][t].w, k4.w, a[g]))));
        }
#pragma unroll
        for (int g = 0; g < ATT_MAXG; ++g) {
            float v = a[g];
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0 && g < ng) sc[g][j] = __fmul_rn(v, scale);
        }
    }
    __syncthreads();
    // per head: chunk max and exp sums (warp g handles heads g, g+4)
    for (int g = warp; g < ng; g += ATT_GLOBAL_THREADS / 32) {
        float m = -INFINITY;
        for (int j = lane; j < nj; j += 32) m = fmaxf(m, sc[g][j]);
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float l = 0.0f;
        for (int j = lane; j < nj; j += 32) {
            const float e = q35_expf(__fsub_rn(sc[g][j], m));
            sc[g][j] = e;
            l += e;
        }
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        if (lane == 0) { red[g][0] = m; red[g][1] = l; }
    }
    __syncthreads();
    // o[g][d] = sum_j e[g][j] * v[j][d]; thread d (D <= 2 * ATT_GLOBAL_THREADS handled by the loop)
    for (int d = threadIdx.x; d < D; d += ATT_GLOBAL_THREADS) {
        float o[ATT_MAXG];
        for (int g = 0; g < ATT_MAXG; ++g) o[g] = 0.0f;
        for (int j = 0; j < nj; ++j) {
            const float v = V[(size_t)j * D + d];
#pragma unroll
            for (int g = 0; g < ATT_MAXG; ++g) o[g] = fmaf(sc[g][j], v, o[g]);
        }
        for (int g = 0; g < ng; ++g) pout(kvh * G + g0 + g)[d] = o[g];
    }
    if (threadIdx.x < ng) {
        pout(kvh * G + g0 + threadIdx.x)[D] = red[threadIdx.x][0];
        pout(kvh * G + g0 + threadIdx.x)[D + 1] = red[threadIdx.x][1];
    }
}

__global__ void attn_combine_kernel(const float *__restrict__ part, int8_t *__restrict__ out_q,
                                    float *__restrict__ out_f, int32_t H, int32_t D, int32_t nchunk) {
    pdl_trigger();
    pdl_wait();
    const int r = blockIdx.x, h = blockIdx.y;
    const float *p = part + ((size_t)r * H + h) * nchunk * (D + 2);
    float M = -INFINITY;
    for (int c = 0; c < nchunk; ++c) M = fmaxf(M, p[(size_t)c * (D + 2) + D]);
    float L = 0.0f;
    for (int c = 0; c < nchunk; ++c) {
        const float m = p[(size_t)c * (D + 2) + D];
        if (m != -INFINITY) L = fmaf(p[(size_t)c * (D + 2) + D + 1], q35_expf(__fsub_rn(m, M)), L);
    }
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float a = 0.0f;
        for (int c = 0; c < nchunk; ++c) {
            const float m = p[(size_t)c * (D + 2) + D];
            if (m != -INFINITY) a = fmaf(p[(size_t)c * (D + 2) + d], q35_expf(__fsub_rn(m, M)), a);
        }
        a = __fdiv_rn(a, L);
        const size_t o = (size_t)r * H * D + (size_t)h * D + d;
        if (out_q) out_q[o] = quant127(a);
        if (out_f) out_f[o] = a;
    }
}

// transformer_layer.f90:212-229 swiglu + the int8 quantization of the down-projection
// input, after the tensor-core gate|up matmul.  y = [R][2F], gate|up columns interleaved:
// gate j at 2j, up j at 2j+1.
__global__ void swiglu_kernel(const float *__restrict__ y, int8_t *__restrict__ out_q,
                              float *__restrict__ out_f, int32_t F, int64_t total) {
    pdl_trigger();
    pdl_wait();
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = t / F, j = t % F;   // gate|up columns interleaved: (gate j, up j) at 2j, 2j+1
        const float g = y[r * 2 * F + 2 * j], u = y[r * 2 * F + 2 * j + 1];
        const float sw = __fdiv_rn(g, __fadd_rn(1.0f, q35_expf(-g)));
        const float h = __fmul_rn(sw, u);
        if (out_q) out_q[t] = quant127(h);
        if (out_f) out_f[t] = h;
    }
}

// llama_model.f90:138-140 LM head: logits(i,j) = dot_product(x_norm(i,:), W(:,j)),
// W stored row-major [vocab][hidden] (the reference's column j contiguous), fused with
// a per-CTA greedy candidate (largest logit, lowest index on ties, sampling.f90:64-83).
constexpr int LMH_THREADS = 256;
// RB: rows per pass over the weights, JW: vocabulary rows a warp takes at once (the model
// runs <1, 1> at batch 1; decode batches run lmhead_rows_kernel below).  Each (row, vocabulary row)
// sum runs over k in the same per-lane order whatever RB and JW are, then the butterfly.
template <int RB, int JW>
__global__ void __launch_bounds__(LMH_THREADS)
lmhead_kernel(const float *__restrict__ xn, const float *__restrict__ W, float *__restrict__ logits,
              float2 *__restrict__ cand, int32_t R, int32_t hidden, int32_t vocab) {
    pdl_trigger();
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t gw = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
    const int64_t nwt = (int64_t)gridDim.x * (blockDim.x >> 5);
    __shared__ float bv[LMH_THREADS / 32][8];
    __shared__ int bi[LMH_THREADS / 32][8];
    float best[8];
    int bidx[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) { best[r] = -FLT_MAX; bidx[r] = 0x7fffffff; }
    for (int64_t jb = gw * JW; jb < vocab; jb += nwt * JW) {
        for (int r0 = 0; r0 < R; r0 += RB) {
            float a[JW][RB];
#pragma unroll
            for (int jj = 0; jj < JW; ++jj)
#pragma unroll
                for (int rr = 0; rr < RB; ++rr) a[jj][rr] = 0.0f;
            // U 512-byte pieces of each weight row in flight per warp, consumed in k order
            constexpr int U = JW == 1 ? 8 : 2;
            for (int k0 = lane * 4; k0 < hidden; k0 += 128 * U) {
                float4 w4[JW][U];
#pragma unroll
                for (int jj = 0; jj < JW; ++jj)
#pragma unroll
                    for (int u = 0; u < U; ++u)
                        w4[jj][u] = (jb + jj < vocab && k0 + 128 * u < hidden)
                                        ? __ldcs(reinterpret_cast<const float4 *>(W + (size_t)(jb + jj) * hidden + k0 + 128 * u))
                                        : make_float4(0.f, 0.f, 0.f, 0.f);   // streamed once
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int k = k0 + 128 * u;
                    if (k >= hidden) break;
#pragma unroll
                    for (int rr = 0; rr < RB; ++rr) {
                        if (r0 + rr < R) {
                            const float4 x4 = *reinterpret_cast<const float4 *>(xn + (size_t)(r0 + rr) * hidden + k);
#pragma unroll
                            for (int jj = 0; jj < JW; ++jj)
                                a[jj][rr] = fmaf(w4[jj][u].x, x4.x, fmaf(w4[jj][u].y, x4.y, fmaf(w4[jj][u].z, x4.z,
                                            fmaf(w4[jj][u].w, x4.w, a[jj][rr]))));
                        }
                    }
                }
            }
#pragma unroll
            for (int jj = 0; jj < JW; ++jj) {
                const int64_t j = jb + jj;
                if (j >= vocab) break;
#pragma unroll
                for (int rr = 0; rr < RB; ++rr) {
                    float v = a[jj][rr];
                    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                    const int row = r0 + rr;
                    if (row < R) {
                        if (lane == 0) logits[(size_t)row * vocab + j] = v;
                        // rows 0..7 keep a per-CTA candidate (the select keeps best[] in registers)
#pragma unroll
                        for (int qq = 0; qq < 8; ++qq)
                            if (qq == row && (v > best[qq] || (v == best[qq] && j < bidx[qq]))) {
                                best[qq] = v;
                                bidx[qq] = (int)j;
                            }
                    }
                }
            }
        }
    }
    // candidates of rows 0..7 per CTA (rows >= 8 are reduced from the logits buffer)
    if (lane == 0)
        for (int r = 0; r < 8; ++r) { bv[warp][r] = best[r]; bi[warp][r] = bidx[r]; }
    __syncthreads();
    if (threadIdx.x < 8 && threadIdx.x < R) {
        const int r = threadIdx.x;
        float v = -FLT_MAX;
        int ix = 0x7fffffff;
        for (int w = 0; w < LMH_THREADS / 32; ++w)
            if (bv[w][r] > v || (bv[w][r] == v && bi[w][r] < ix)) { v = bv[w][r]; ix = bi[w][r]; }
        cand[(size_t)r * gridDim.x + blockIdx.x] = make_float2(v, __int_as_float(ix));
    }
}

// The LM head for decode batches: a CTA takes blocks of 32 vocabulary rows (8 warps x
// LMB_JW) and, for each pass of LMB_RB rows, stages the rows' activations in shared memory
// one LMB_KC-wide chunk of k at a time for all its warps (a warp reading them from L2 per
// weight load moved several times the weights' bytes).  A lane still visits k = 4 lane,
// 4 lane + 128, ... in order and the sums end in the same butterfly, so every logit equals
// lmhead_kernel's.
constexpr int LMB_RB = 8, LMB_JW = 4, LMB_KC = 2048, LMB_U = 2;
__global__ void __launch_bounds__(LMH_THREADS)
lmhead_rows_kernel(const float *__restrict__ xn, const float *__restrict__ W, float *__restrict__ logits,
                   float2 *__restrict__ cand, int32_t R, int32_t hidden, int32_t vocab) {
    extern __shared__ __align__(16) float4 xs4[];   // [LMB_RB][LMB_KC / 4]
    __shared__ float bv[LMH_THREADS / 32][8];
    __shared__ int bi[LMH_THREADS / 32][8];
    pdl_trigger();
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int NW = LMH_THREADS / 32;
    const int64_t nblk = ((int64_t)vocab + NW * LMB_JW - 1) / (NW * LMB_JW);
    const float4 *xn4 = reinterpret_cast<const float4 *>(xn);
    const int h4 = hidden / 4;
    float best[8];
    int bidx[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) { best[r] = -FLT_MAX; bidx[r] = 0x7fffffff; }
    for (int64_t blk = blockIdx.x; blk < nblk; blk += gridDim.x) {
        const int64_t jb = (blk * NW + warp) * LMB_JW;   // this warp's vocabulary rows
        for (int r0 = 0; r0 < R; r0 += LMB_RB) {
            float a[LMB_JW][LMB_RB];
#pragma unroll
            for (int jj = 0; jj < LMB_JW; ++jj)
#pragma unroll
                for (int rr = 0; rr < LMB_RB; ++rr) a[jj][rr] = 0.0f;
            for (int kc = 0; kc < hidden; kc += LMB_KC) {
                const int kn = min(LMB_KC, hidden - kc), kn4 = kn / 4;
                __syncthreads();   // every warp is done with the previous chunk
                for (int i = threadIdx.x; i < LMB_RB * kn4; i += LMH_THREADS) {
                    const int rr = i / kn4, q4 = i - rr * kn4;
                    xs4[rr * (LMB_KC / 4) + q4] = (r0 + rr < R) ? xn4[(size_t)(r0 + rr) * h4 + kc / 4 + q4]
                                                                : make_float4(0.f, 0.f, 0.f, 0.f);
                }
                __syncthreads();
                for (int k0 = lane * 4; k0 < kn; k0 += 128 * LMB_U) {
                    float4 w4[LMB_JW][LMB_U];
#pragma unroll
                    for (int jj = 0; jj < LMB_JW; ++jj)
#pragma unroll
                        for (int u = 0; u < LMB_U; ++u)
                            w4[jj][u] = (jb + jj < vocab && k0 + 128 * u < kn)
                                            ? __ldcs(reinterpret_cast<const float4 *>(W + (size_t)(jb + jj) * hidden + kc + k0 + 128 * u))
                                            : make_float4(0.f, 0.f, 0.f, 0.f);   // streamed once
#pragma unroll
                    for (int u = 0; u < LMB_U; ++u) {
                        const int k = k0 + 128 * u;
                        if (k >= kn) break;
#pragma unroll
                        for (int rr = 0; rr < LMB_RB; ++rr) {
                            if (r0 + rr < R) {
                                const float4 x4 = xs4[rr * (LMB_KC / 4) + k / 4];
#pragma unroll
                                for (int jj = 0; jj < LMB_JW; ++jj)
                                    a[jj][rr] = fmaf(w4[jj][u].x, x4.x, fmaf(w4[jj][u].y, x4.y, fmaf(w4[jj][u].z, x4.z,
                                                fmaf(w4[jj][u].w, x4.w, a[jj][rr]))));
                            }
                        }
                    }
                }
            }
#pragma unroll
            for (int jj = 0; jj < LMB_JW; ++jj) {
                const int64_t j = jb + jj;
                if (j >= vocab) break;
#pragma unroll
                for (int rr = 0; rr < LMB_RB; ++rr) {
                    float v = a[jj][rr];
                    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                    const int row = r0 + rr;
                    if (row < R) {
                        if (lane == 0) logits[(size_t)row * vocab + j] = v;
#pragma unroll
                        for (int qq = 0; qq < 8; ++qq)
                            if (qq == row && (v > best[qq] || (v == best[qq] && j < bidx[qq]))) {
                                best[qq] = v;
                                bidx[qq] = (int)j;
                            }
                    }
                }
            }
        }
    }
    // candidates of rows 0..7 per CTA (rows >= 8 are reduced from the logits buffer)
    if (lane == 0)
        for (int r = 0; r < 8; ++r) { bv[warp][r] = best[r]; bi[warp][r] = bidx[r]; }
    __syncthreads();
    if (threadIdx.x < 8 && threadIdx.x < R) {
        const int r = threadIdx.x;
        float v = -FLT_MAX;
        int ix = 0x7fffffff;
        for (int w = 0; w < NW; ++w)
            if (bv[w][r] > v || (bv[w][r] == v && bi[w][r] < ix)) { v = bv[w][r]; ix = bi[w][r]; }
        cand[(size_t)r * gridDim.x + blockIdx.x] = make_float2(v, __int_as_float(ix));
    }
}

// greedy token per row (1-based), from the per-CTA candidates (rows < 8) or by a scan of
// the row's logits (rows >= 8); lowest index wins ties.  idx0 is the global index of the
// first local logit (vocab-split LM head); pair_out receives (value, global index).
__global__ void argmax_kernel(const float2 *__restrict__ cand, int32_t ncand, const float *__restrict__ logits,
                              int32_t vocab, int32_t idx0, int32_t *__restrict__ tok_out,
                              float2 *__restrict__ pair_out) {
    __shared__ float sv[256];
    __shared__ int si[256];
    pdl_trigger();
    pdl_wait();
    const int r = blockIdx.x;
    float v = -FLT_MAX;
    int ix = 0x7fffffff;
    if (r < 8) {
        for (int c = threadIdx.x; c < ncand; c += blockDim.x) {
            const float2 e = cand[(size_t)r * ncand + c];
            const int ei = __float_as_int(e.y);
            if (e.x > v || (e.x == v && ei < ix)) { v = e.x; ix = ei; }
        }
    } else {
        for (int j = threadIdx.x; j < vocab; j += blockDim.x) {
            const float e = logits[(size_t)r * vocab + j];
            if (e > v) { v = e; ix = j; }
        }
    }
    sv[threadIdx.x] = v;
    si[threadIdx.x] = ix;
    __syncthreads();
    for (int s = blockDim.x / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s) {
            const float ov = sv[threadIdx.x + s];
            const int oi = si[threadIdx.x + s];
            if (ov > sv[threadIdx.x] || (ov == sv[threadIdx.x] && oi < si[threadIdx.x])) {
                sv[threadIdx.x] = ov;
                si[threadIdx.x] = oi;
            }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        if (tok_out) tok_out[r] = idx0 + si[0] + 1;
        if (pair_out) pair_out[r] = make_float2(sv[0], __int_as_float(idx0 + si[0]));
    }
}

// greedy over the ranks' candidates [world][R] (lowest global index on ties)
__global__ void merge_argmax_kernel(const float2 *__restrict__ pairs, int32_t world, int32_t R,
                                    int32_t *__restrict__ tok_out) {
    pdl_trigger();
    pdl_wait();
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= R) return;
    float v = -FLT_MAX;
    int ix = 0x7fffffff;
    for (int w = 0; w < world; ++w) {
        const float2 e = pairs[(size_t)w * R + r];
        const int ei = __float_as_int(e.y);
        if (e.x > v || (e.x == v && ei < ix)) { v = e.x; ix = ei; }
    }
    tok_out[r] = ix + 1;
}

// x += (float(C) + offset) * scale after the all-reduce of a row-split matmul
// (matmul_3p5bit_dynamic.f90:80 / matmul_int4_groq.f90:151, then the residual add of
// transformer_layer.f90:550 / :557)
__global__ void dequant_residual_kernel(const int32_t *__restrict__ C, const float *__restrict__ scales,
                                        const float *__restrict__ offsets, float *__restrict__ x, int32_t N,
                                        int64_t total) {
    pdl_trigger();
    pdl_wait();
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = t % N;
        const float f = __int2float_rn(C[t]);
        const float y = offsets ? __fmul_rn(__fadd_rn(f, offsets[j]), scales[j]) : __fmul_rn(f, scales[j]);
        x[t] = __fadd_rn(x[t], y);
    }
}

// cache_pos[seq] += n for the sequences of a forward (transformer_layer.f90:424-426)
__global__ void advance_kernel(int32_t *cache_pos, const int32_t *seqs, int32_t nseq, int32_t n) {
    pdl_wait();
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t < nseq) cache_pos[seqs[t]] += n;
}

// ---------------------------------------------------------------------------------------
static int grid_1d(int64_t n, int threads) { return (int)std::min<int64_t>(ceil_div(n, threads), 148 * 16); }

int launch_embed(const int32_t *ids, const float *E, float *x, int R, int hidden, int vocab, int *err,
                 cudaStream_t s) {
    if (hidden % 4) return set_error(Q35_ERR_INVALID, "embed: hidden must be a multiple of 4");
    return launch_pdl(embed_kernel, dim3(R, (unsigned)ceil_div(hidden / 4, 256)), dim3(256), 0, s, ids, E, x, hidden,
                      vocab, err);
}

int launch_rmsnorm(const float *x, const float *w, float *out, int8_t *q, int R, int dim, float eps,
                   cudaStream_t s) {
    if (dim % 4) return set_error(Q35_ERR_INVALID, "rmsnorm: dim must be a multiple of 4");
    if (R <= 0) return Q35_OK;
    static int sms[64] = {0};
    int dev = 0;
    Q35_CUDA_TRY(cudaGetDevice(&dev));
    const int di = dev >= 0 && dev < 64 ? dev : 0;
    if (!sms[di]) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
        sms[di] = v;
    }
    // few rows: 4 * K4 CTAs per row, one element per thread (K4 float4s per thread in the sum)
    const int K4 = (int)ceil_div((int64_t)(dim / 4), NORM_THREADS);
    const int split = (K4 <= NORM_KMAX && (int64_t)R * 4 * K4 <= sms[di]) ? 4 * K4 : 1;
    return launch_pdl(rmsnorm_kernel, dim3(R, split), dim3(NORM_THREADS), 0, s, x, w, out, q, dim, eps, split);
}

int launch_rope_kv(const float *yqkv, float *q, float *kc, float *vc, const int32_t *row_seq,
                   const int32_t *row_i, const int32_t *cache_pos, const float2 *cs, int layer,
                   int n_layers, int R, int H, int KVH, int D, int max_seq, int rope_mode, int *err,
                   cudaStream_t s) {
    return launch_pdl(rope_kv_kernel, dim3(R, H + KVH), dim3(64), 0, s, yqkv, q, kc, vc, row_seq, row_i,
                      cache_pos, cs, layer, n_layers, H, KVH, D, max_seq, rope_mode, err);
}

int attn_part_floats(int R, int H, int D, int max_seq) {
    return R * H * ((max_seq + ATT_CHUNK - 1) / ATT_CHUNK) * (D + 2);
}

int launch_attention(const float *q, const float *kc, const float *vc, float *part, int8_t *out_q, float *out_f,
                     const int32_t *row_seq, const int32_t *row_i, const int32_t *cache_pos, int layer, int n_layers,
                     int R, int H, int KVH, int D, int max_seq, int *err, cudaStream_t s, bool shared_rows) {
    if (D % 128 || D > 256) return set_error(Q35_ERR_INVALID, "attention: head_dim must be 128 or 256");
    const int nchunk = (max_seq + ATT_CHUNK - 1) / ATT_CHUNK;
    if (nchunk > ATT_MAX_CHUNKS) return set_error(Q35_ERR_INVALID, "attention: max_seq above 8192");
    const int G = H / KVH, gparts = (G + ATT_MAXG - 1) / ATT_MAXG;
    if (R > 1 && shared_rows) {   // the rows of one sequence (prefill): chunks shared through L1
        auto pk = D == 128 ? attn_partial_global_kernel<1> : attn_partial_global_kernel<2>;
        int st = launch_pdl(pk, dim3(R, KVH * gparts, nchunk), dim3(ATT_GLOBAL_THREADS), 0, s, q, kc, vc, part,
                            row_seq, row_i, cache_pos, (int32_t)layer, (int32_t)n_layers, (int32_t)H, (int32_t)KVH,
                            (int32_t)D, (int32_t)max_seq, (int32_t)nchunk);
        if (st) return st;
        return launch_pdl(attn_combine_kernel, dim3(R, H), dim3(128), 0, s, part, out_q, out_f, (int32_t)H, (int32_t)D,
                          (int32_t)nchunk);
    }
    if (R > 1) {   // rows give the parallelism: light CTAs, partials in global memory
        auto pk = D == 128 ? attn_partial_kernel<1> : attn_partial_kernel<2>;
        const size_t psmem = (size_t)2 * ATT_CHUNK * D * sizeof(float) + 16;
        static bool pconfigured[2][64] = {};
        int st = smem_limit_once(pconfigured[D / 128 - 1], pk, psmem);
        if (st) return st;
        st = launch_pdl(pk, dim3(R, KVH * gparts, nchunk), dim3(ATT1_THREADS), psmem, s, q, kc, vc, part, row_seq,
                            row_i, cache_pos, (int32_t)layer, (int32_t)n_layers, (int32_t)H, (int32_t)KVH,
                            (int32_t)max_seq, (int32_t)nchunk, err);
        if (st) return st;
        return launch_pdl(attn_combine_kernel, dim3(R, H), dim3(128), 0, s, part, out_q, out_f, (int32_t)H, (int32_t)D,
                          (int32_t)nchunk);
    }
    // CTAs per cluster: ATT_CS, fewer when the cache has fewer chunks (short contexts: no
    // CTA without a chunk holds an SM)
    const int cs = std::min(ATT_CS, nchunk);
    const int slots = (nchunk + cs - 1) / cs;   // chunks per CTA, at most
    // double-buffered stages only where a CTA has a next chunk to stream in; smaller CTAs
    // share an SM (MHA at short contexts: many clusters, one chunk per CTA)
    const int nb = (D == 128 && slots > 1) ? 2 : 1;
    const bool flex = cs < ATT_CS || nb != (D == 128 ? 2 : 1) || H / KVH < ATT_MAXG;
    const size_t smem_max = 227 * 1024 - 8192;
    // merge buffer: ceil(gp / cs) merged heads per CTA x every chunk
    const int gp = flex ? std::min(G, ATT_MAXG) : ATT_MAXG;
    const int32_t mbf = ((gp + cs - 1) / cs) * nchunk * (D + 2);
    size_t smem = ((size_t)nb * 2 * ATT_CHUNK * D + (size_t)mbf) * sizeof(float) + 16;
    if (smem > 227 * 1024) return set_error(Q35_ERR_INVALID, "attention: max_seq too long for head_dim 256");
    // the scores' lane partials in shared memory where they fit (head_dim 128, max_seq up to
    // 2048); otherwise the same sums by warp shuffles
    const size_t part_bytes = sizeof(float) * ATT_CHUNK * gp * ATT_PSTR;
    const int32_t use_part = (D == 128 && smem + part_bytes <= smem_max) ? 1 : 0;
    if (use_part) smem += part_bytes;
    auto kern = D == 128 ? (flex ? attn_kernel<1, true> : attn_kernel<1, false>)
                         : (flex ? attn_kernel<2, true> : attn_kernel<2, false>);
    static bool configured[4][64] = {};
    const int ki = (D / 128 - 1) * 2 + (flex ? 1 : 0);
    int st = smem_limit_once(configured[ki], kern, smem_max);
    if (st) return st;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(R, KVH * gparts * cs);
    cfg.blockDim = dim3(ATT1_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = cs;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    Q35_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, q, kc, vc, out_q, out_f, row_seq, row_i, cache_pos, (int32_t)layer,
                                    (int32_t)n_layers, (int32_t)H, (int32_t)KVH, (int32_t)max_seq, mbf,
                                    (int32_t)nb, (int32_t)cs, use_part, err));
    return Q35_OK;
}

int launch_swiglu(const float *y, int8_t *out_q, float *out_f, int R, int F, cudaStream_t s) {
    const int64_t total = (int64_t)R * F;
    return launch_pdl(swiglu_kernel, dim3(grid_1d(total, 256)), dim3(256), 0, s, y, out_q, out_f, F, total);
}

int lmhead_grid(int dev) {
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms * 4;
}

int launch_lmhead(const float *xn, const float *W, float *logits, float2 *cand, int32_t *tok, float2 *pairs,
                  int idx0, int R, int hidden, int vocab, int grid, cudaStream_t s) {
    int st = Q35_OK;
    if (R == 1) {
        st = launch_pdl(lmhead_kernel<1, 1>, dim3(grid), dim3(LMH_THREADS), 0, s, xn, W, logits, cand, R, hidden,
                        vocab);
    } else {
        // decode batches: the activations of a pass staged per CTA; as many CTAs as two per
        // SM hold (the candidates buffer has room for `grid`), at most one per block of
        // vocabulary rows
        const size_t smem = sizeof(float) * LMB_RB * LMB_KC;
        static bool configured[64] = {};
        st = smem_limit_once(configured, lmhead_rows_kernel, smem);
        if (st) return st;
        const int64_t nblk = ((int64_t)vocab + (LMH_THREADS / 32) * LMB_JW - 1) / ((LMH_THREADS / 32) * LMB_JW);
        grid = (int)std::max<int64_t>(1, std::min<int64_t>(grid / 2, nblk));
        st = launch_pdl(lmhead_rows_kernel, dim3(grid), dim3(LMH_THREADS), smem, s, xn, W, logits, cand, R, hidden,
                        vocab);
    }
    if (st) return st;
    return launch_pdl(argmax_kernel, dim3(R), dim3(256), 0, s, (const float2 *)cand, grid, (const float *)logits,
                      vocab, idx0, tok, pairs);
}

int launch_merge_argmax(const float2 *pairs, int world, int R, int32_t *tok, cudaStream_t s) {
    return launch_pdl(merge_argmax_kernel, dim3((R + 127) / 128), dim3(128), 0, s, pairs, world, R, tok);
}

int launch_dequant_residual(const int32_t *C, const float *scales, const float *offsets, float *x, int R, int N,
                            cudaStream_t s) {
    const int64_t total = (int64_t)R * N;
    return launch_pdl(dequant_residual_kernel, dim3(grid_1d(total, 256)), dim3(256), 0, s, C, scales, offsets, x, N,
                      total);
}

int launch_advance(int32_t *cache_pos, const int32_t *seqs, int nseq, int n, cudaStream_t s) {
    return launch_pdl(advance_kernel, dim3((nseq + 127) / 128), dim3(128), 0, s, cache_pos, seqs, nseq, n);
}

}  // namespace q35
