// q35_sample.cu -- the sampling module (sampling.f90) on the device: greedy, temperature,
// top-k and top-p (nucleus) sampling fused into one kernel, one CTA of 1024 threads per
// row of logits (thread t owns entries [32t, 32t+32)).
//
// Semantics follow sampling.f90:
//  * sample_greedy (:64-83): first index of the maximum (strict >), 1-based.
//  * sample_temperature (:88-118): logits / T when T > 0 (apply_temperature, :25-29),
//    softmax with max subtraction and the sum > 0 guard (:35-59), then the first index i
//    with u <= cumsum(i) over all i; the last token when there is none.
//  * sample_top_k (:123-176): kth = the k-th largest logit counted with multiplicity (k
//    rounds of "max, mask its first occurrence", :139-147; -huge when k <= 0 or k > vocab);
//    logits below kth become -huge (:150-156); softmax; the first i with probs(i) > 0 and
//    u <= the running sum over those i (:164-175).  No temperature.
//  * sample_top_p (:181-259): probs = softmax(logits); threshold = the descending-sorted
//    probability at which the running sum first reaches p (:220-230; 0 when it never
//    does); logits whose probability is below the threshold become -huge (:233-239);
//    softmax again; sampled as top-k (:247-258).
// random_number is replaced by a uniform u in [0,1) that the caller passes, or that the
// kernel draws per sequence from the counter-based generator (seed, SAMPLE_STREAM + seq,
// draw count): u = (top 24 bits of the draw) * 2^-24.
//
// Arithmetic.  The softmax normaliser is an fp32 sum in a fixed order (the reference's
// loop is sequential; this one is blocked, restated by the oracle's order-1 sampler):
//   T_t = thread t's entries summed one at a time from 0
//   W_w = T_32w + ... + T_32w+31, one at a time from 0
//   Q_0 = 0, Q_w+1 = Q_w + W_w;  sum = Q_32
// Every exponential is q35_expf (q35_expf.h).  The running sums over probabilities (the
// top-p threshold, the draw) are exact integer sums of the probabilities in fixed point,
// fx(p) = floor(p * 2^40) (64-bit), compared with fx(u) and fx(top_p): they equal the
// reference's fp32 running sums up to rounding, do not depend on the order of addition,
// and so run as parallel scans.  The top-p threshold is the largest probability v with
// sum over {p_i >= v} of fx(p_i) >= fx(top_p) -- the sorted running sum's crossing value
// -- found by a radix descent over the probabilities' bit patterns (no sort).
// A row is loaded into shared memory with coalesced reads; each thread then takes its
// chunk (one pad float every 32 entries keeps those reads free of bank conflicts).
#include <cfloat>
#include <cstring>

#include "q35_expf.h"
#include "q35_internal.cuh"

namespace q35 {
namespace {

constexpr int SNT = 1024;                 // threads per row
constexpr int SCH = 32;                   // entries per thread
constexpr int SNW = SNT / 32;
constexpr int SMAXV = SNT * SCH;          // 32768: largest vocabulary
constexpr uint64_t SAMPLE_STREAM = 0x53414D0000000000ull;

__host__ __device__ inline int pidx(int i) { return i + (i >> 5); }

struct SampleShared {
    float W[SNW];
    float Q[SNW + 1];
    float redf[SNW];
    int redi[SNW];
    unsigned long long mhist[256];
    unsigned long long wsum[SNW];
    unsigned long long carry;
    unsigned lo, hi;
};

constexpr float FX_SCALE = 1099511627776.0f;   // 2^40

// fx(p) = floor(p * 2^40) for p >= 0 (0 for p <= 0 or NaN, saturating above 2^64)
__device__ __forceinline__ unsigned long long fx(float p) {
    return p > 0.0f ? __float2ull_rz(p * FX_SCALE) : 0ull;
}

// exclusive block scan of 64-bit integers (order free: exact)
__device__ unsigned long long scan_u64(SampleShared &sh, unsigned long long v, unsigned long long *total) {
    const int t = threadIdx.x, w = t >> 5, l = t & 31;
    unsigned long long incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long n = __shfl_up_sync(0xffffffffu, incl, o);
        if (l >= o) incl += n;
    }
    if (l == 31) sh.wsum[w] = incl;
    __syncthreads();
    if (w == 0) {
        const unsigned long long mine = sh.wsum[l];
        unsigned long long wi = mine;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned long long n = __shfl_up_sync(0xffffffffu, wi, o);
            if (l >= o) wi += n;
        }
        sh.wsum[l] = wi - mine;          // exclusive
        if (l == 31) sh.carry = wi;
    }
    __syncthreads();
    const unsigned long long ex = sh.wsum[w] + incl - v;
    if (total) *total = sh.carry;
    __syncthreads();
    return ex;
}

__device__ __forceinline__ uint64_t smix(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

// the fixed-order sum of every thread's chunk sum Tt; *prefix gets the running sum before
// thread t's chunk.  All threads call it.
__device__ float ordered_scan(SampleShared &sh, float Tt, float *prefix) {
    const int t = threadIdx.x, w = t >> 5, l = t & 31;
    float Ww = 0.0f;                       // W_w, the same in every lane
#pragma unroll
    for (int i = 0; i < 32; ++i) Ww = __fadd_rn(Ww, __shfl_sync(0xffffffffu, Tt, i));
    if (l == 0) sh.W[w] = Ww;
    __syncthreads();
    if (w == 0) {
        const float mine = sh.W[l];
        float q = 0.0f;                    // lane l: Q_l = W_0 + ... + W_l-1
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const float v = __shfl_sync(0xffffffffu, mine, i);
            if (i < l) q = __fadd_rn(q, v);
        }
        sh.Q[l] = q;
        if (l == 31) sh.Q[SNW] = __fadd_rn(q, mine);
    }
    __syncthreads();
    if (prefix) {
        float p = sh.Q[w];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const float v = __shfl_sync(0xffffffffu, Tt, i);
            if (i < l) p = __fadd_rn(p, v);
        }
        *prefix = p;
    }
    const float total = sh.Q[SNW];
    __syncthreads();
    return total;
}

__device__ float block_max(SampleShared &sh, float v) {
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31) == 0) sh.redf[threadIdx.x >> 5] = v;
    __syncthreads();
    float m = sh.redf[threadIdx.x & 31];
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    __syncthreads();
    return m;
}

__device__ int block_min_int(SampleShared &sh, int v) {
    for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31) == 0) sh.redi[threadIdx.x >> 5] = v;
    __syncthreads();
    int m = sh.redi[threadIdx.x & 31];
    for (int o = 16; o > 0; o >>= 1) m = min(m, __shfl_xor_sync(0xffffffffu, m, o));
    __syncthreads();
    return m;
}

// order-preserving key of a float (larger float, larger key)
__device__ __forceinline__ unsigned fkey(float f) {
    const unsigned b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float fkey_inv(unsigned k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

__device__ unsigned block_max_u(SampleShared &sh, unsigned v) {
    v = __reduce_max_sync(0xffffffffu, v);
    if ((threadIdx.x & 31) == 0) sh.redi[threadIdx.x >> 5] = (int)v;
    __syncthreads();
    const unsigned m = __reduce_max_sync(0xffffffffu, (unsigned)sh.redi[threadIdx.x & 31]);
    __syncthreads();
    return m;
}

// The largest key v among this CTA's entries whose weight W(v) = sum of the weights of the
// entries with key >= v reaches target, given lo <= v <= hi, mass above hi = 0 and
// W(lo) >= target >= 1.  A radix descent: each level cuts [lo, hi] into <= 256
// power-of-two bins (integer weights, so the bins' sums are exact in any order) and keeps
// the highest bin whose weight, with everything above it, reaches the target.
// kw(j, key, w) gives thread entry j's key and weight (j < nj); COUNT: every weight is 1.
template <bool COUNT, typename KW>
__device__ unsigned descend(SampleShared &sh, KW kw, int nj, unsigned lo, unsigned hi,
                            unsigned long long target) {
    const int t = threadIdx.x;
    unsigned long long carry = 0;
    // each level leaves a range below 2^sft <= range / 128, so a 32-bit key range takes
    // at most 5 levels; the cap only bounds the loop
    for (int level = 0; lo < hi && level < 8; ++level) {
        const unsigned range = hi - lo;
        int sft = 0;
        while ((range >> sft) >= 256u) ++sft;
        const int nb = (int)(range >> sft) + 1;
        for (int i = t; i < 256; i += SNT) sh.mhist[i] = 0ull;
        __syncthreads();
        if (COUNT) {
            // unit weights: lanes with the same bin add once (logits crowd a few bins)
            for (int j = 0; j < SCH; ++j) {
                unsigned k = 0u;
                unsigned long long w = 0ull;
                if (j < nj) kw(j, k, w);
                const bool in = j < nj && k >= lo && k <= hi;
                const unsigned bin = in ? (k - lo) >> sft : 256u;
                const unsigned same = __match_any_sync(0xffffffffu, bin);
                if (in && (threadIdx.x & 31) == (unsigned)(__ffs(same) - 1))
                    atomicAdd(&sh.mhist[bin], (unsigned long long)__popc(same));
            }
        } else {
            for (int j = 0; j < nj; ++j) {
                unsigned k;
                unsigned long long w;
                kw(j, k, w);
                if (w != 0ull && k >= lo && k <= hi) atomicAdd(&sh.mhist[(k - lo) >> sft], w);
            }
        }
        __syncthreads();
        if (t < 32) {
            // lane l: bins nb-1-8l .. nb-8-8l (descending); weight above them by a scan
            unsigned long long m[8], mine = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int d = nb - 1 - 8 * t - i;
                m[i] = d >= 0 ? sh.mhist[d] : 0ull;
                mine += m[i];
            }
            unsigned long long incl = mine;
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned long long n = __shfl_up_sync(0xffffffffu, incl, o);
                if (t >= o) incl += n;
            }
            unsigned long long c = carry + incl - mine;
            if (c < target && carry + incl >= target) {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int d = nb - 1 - 8 * t - i;
                    if (d >= 0 && c + m[i] >= target) {
                        const unsigned b0 = lo + ((unsigned)d << sft);
                        sh.lo = b0;
                        sh.hi = min(hi, b0 + ((1u << sft) - 1u));
                        sh.carry = c;
                        break;
                    }
                    c += m[i];
                }
            }
        }
        __syncthreads();
        lo = sh.lo;
        hi = sh.hi;
        carry = sh.carry;
        __syncthreads();
    }
    return lo;
}

struct SampleParams {
    const float *logits;      // element (row r, token g): logits[((g / Vl) * Rtot + r) * Vl + g % Vl]
    int32_t Vl, Rtot, V;      // Vl: entries per block (the vocabulary of one TP rank)
    int32_t row0;             // rows row0 .. row0 + gridDim.x - 1 are sampled
    int32_t mode, top_k;
    float temperature, top_p;
    const float *u;           // per sampled row, or nullptr: drawn per sequence
    uint64_t seed;
    const int32_t *row_seq;   // sequence of a row (nullptr: the row index)
    int32_t row_seq0;         // row_seq index of row 0
    int32_t *draws;           // per sequence draw counters (u == nullptr)
    int32_t *tokens;          // 1-based token per sampled row
};

__global__ void __launch_bounds__(SNT, 1) sample_kernel(SampleParams P) {
    extern __shared__ float srt[];
    __shared__ SampleShared sh;
    const int t = threadIdx.x;
    const int r = P.row0 + blockIdx.x;
    const int base = t * SCH;
    const int V = P.V;

    // coalesced loads of the row into shared memory, then each thread's chunk
    for (int blk = 0, g0 = 0; g0 < V; ++blk, g0 += P.Vl) {
        const float *src = P.logits + ((size_t)blk * P.Rtot + r) * P.Vl;
        for (int jl = t; jl < P.Vl; jl += SNT) srt[pidx(g0 + jl)] = src[jl];
    }
    __syncthreads();
    // thread t's entries live in shared memory: X(j) is entry base + j (valid for
    // base + j < V); logits, then exponentials
#define X(j) srt[pidx(base + (j))]
    const int nj = max(0, min(SCH, V - base));

    if (P.mode == Q35_SAMPLE_GREEDY) {
        float bv = -INFINITY;
        int bi = V;
        for (int j = 0; j < nj; ++j)
            if (bi == V || X(j) > bv) { bv = X(j); bi = base + j; }
        const float m = block_max(sh, bi < V ? bv : -INFINITY);
        const int first = block_min_int(sh, (bi < V && bv == m) ? bi : V);
        if (t == 0) P.tokens[blockIdx.x] = (first < V ? first : 0) + 1;
        return;
    }

    // the uniform draw of this row
    float u = 0.0f;
    if (P.u) {
        u = P.u[blockIdx.x];
    } else {
        const int seq = P.row_seq ? P.row_seq[P.row_seq0 + r] : r;
        const int n = P.draws[seq];
        const uint64_t key = smix(P.seed ^ smix(SAMPLE_STREAM + (uint64_t)seq + 0x632BE59BD9B4E019ull));
        const uint64_t z = smix(key + (uint64_t)n * 0x9E3779B97F4A7C15ull);
        u = (float)(uint32_t)(z >> 40) * 0x1p-24f;
        __syncthreads();   // every thread has read the counter
        if (t == 0) P.draws[seq] = n + 1;
    }

    if (P.mode == Q35_SAMPLE_TEMPERATURE && P.temperature > 0.0f)
        for (int j = 0; j < nj; ++j) X(j) = __fdiv_rn(X(j), P.temperature);
    if (P.mode == Q35_SAMPLE_TOP_K) {
        float kth = -FLT_MAX;
        if (P.top_k >= 1 && P.top_k <= V) {
            unsigned kmax = 0u, kmin = 0u;
            for (int j = 0; j < nj; ++j) {
                const unsigned k = fkey(X(j));
                kmax = max(kmax, k);
                kmin = max(kmin, ~k);
            }
            kmax = block_max_u(sh, kmax);
            kmin = ~block_max_u(sh, kmin);
            const unsigned key = descend<true>(
                sh, [&](int j, unsigned &k, unsigned long long &w) { k = fkey(X(j)); w = 1ull; }, nj, kmin, kmax,
                (unsigned long long)P.top_k);
            kth = fkey_inv(key);
        }
        for (int j = 0; j < nj; ++j)
            if (X(j) < kth) X(j) = -FLT_MAX;
    }
    // softmax (:35-59); the entries become the exponentials, probabilities are formed on demand
    float mloc = -INFINITY;
    for (int j = 0; j < nj; ++j) mloc = fmaxf(mloc, X(j));
    const float mx = block_max(sh, mloc);
    float Tt = 0.0f;
    for (int j = 0; j < nj; ++j) {
        const float e = q35_expf(__fsub_rn(X(j), mx));
        X(j) = e;
        Tt = __fadd_rn(Tt, e);
    }
    float sum = ordered_scan(sh, Tt, nullptr);
    const float uniform = __fdiv_rn(1.0f, (float)V);
#define Q35_PROB(j) (sum > 0.0f ? __fdiv_rn(X(j), sum) : uniform)

    if (P.mode == Q35_SAMPLE_TOP_P) {
        // the entries become the probabilities
        float pmax = 0.0f, pmin = INFINITY;
        unsigned long long own = 0;
        for (int j = 0; j < nj; ++j) {
            const float pj = Q35_PROB(j);
            X(j) = pj;
            pmax = fmaxf(pmax, pj);
            pmin = fminf(pmin, pj);
            own += fx(pj);
        }
        pmax = block_max(sh, pmax);
        pmin = -block_max(sh, -pmin);
        unsigned long long total = 0;
        scan_u64(sh, own, &total);
        // threshold: the largest probability v whose fixed-point mass (the probabilities
        // >= v) reaches fx(p); bit patterns of probabilities (>= 0) order like the values
        const unsigned long long target = fx(P.top_p);
        float thr;
        if (!(P.top_p == P.top_p) || total < target)
            thr = 0.0f;                                   // never reached: keep everything
        else if (target == 0ull)
            thr = pmax;                                   // p <= 0: the first entry reaches it
        else
            thr = __uint_as_float(descend<false>(
                sh,
                [&](int j, unsigned &k, unsigned long long &w) {
                    const float pj = X(j);
                    k = __float_as_uint(pj);
                    w = fx(pj);
                },
                nj, __float_as_uint(pmin), __float_as_uint(pmax), target));
        // masked logits -> -huge and softmax again: the kept maximum is the old one, so a
        // kept entry's exponential is the first pass's (recomputed from the logits, which
        // top-p does not scale) and a masked one is exp(-huge - max) = 0
        const float e_masked = q35_expf(__fsub_rn(-FLT_MAX, mx));
        int blk = base / P.Vl, jl = base - blk * P.Vl;
        Tt = 0.0f;
        for (int j = 0; j < nj; ++j) {
            float e = e_masked;
            if (X(j) >= thr) e = q35_expf(__fsub_rn(P.logits[((size_t)blk * P.Rtot + r) * P.Vl + jl], mx));
            X(j) = e;
            Tt = __fadd_rn(Tt, e);
            if (++jl == P.Vl) { ++blk; jl = 0; }
        }
        sum = ordered_scan(sh, Tt, nullptr);
    }

    // draw: the first i (with probs(i) > 0 unless temperature mode) whose running sum
    // reaches u, the sums exact in fixed point
    const bool all = P.mode == Q35_SAMPLE_TEMPERATURE;
    unsigned long long own = 0;
    for (int j = 0; j < nj; ++j) {
        const float pj = Q35_PROB(j);
        X(j) = pj;
        own += fx(pj);
    }
    unsigned long long acc = scan_u64(sh, own, nullptr);
    const unsigned long long ufx = fx(u);
    int hit = V;
    for (int j = 0; j < nj; ++j) {
        const float pj = X(j);
        acc += fx(pj);
        if ((all || pj > 0.0f) && ufx <= acc) { hit = base + j; break; }
    }
#undef Q35_PROB
#undef X
    const int first = block_min_int(sh, hit);
    if (t == 0) P.tokens[blockIdx.x] = (first < V ? first : V - 1) + 1;
}

}  // namespace

int sample_check(int mode, int V) {
    if (mode < Q35_SAMPLE_GREEDY || mode > Q35_SAMPLE_TOP_P) return set_error(Q35_ERR_INVALID, "sampling: unknown mode");
    if (V < 1 || V > SMAXV) return set_error(Q35_ERR_INVALID, "sampling: vocabulary must be 1..32768");
    return Q35_OK;
}

int launch_sample(const SampleRows &a, cudaStream_t s) {
    int st = sample_check(a.mode, a.V);
    if (st) return st;
    if (a.rows < 1) return Q35_OK;
    if (a.Vl < 1 || a.V % a.Vl) return set_error(Q35_ERR_INVALID, "sampling: vocabulary blocks");
    SampleParams P;
    P.logits = a.logits;
    P.Vl = a.Vl;
    P.Rtot = a.Rtot;
    P.V = a.V;
    P.row0 = a.row0;
    P.mode = a.mode;
    P.top_k = a.top_k;
    P.temperature = a.temperature;
    P.top_p = a.top_p;
    P.u = a.u;
    P.seed = a.seed;
    P.row_seq = a.row_seq;
    P.row_seq0 = a.row_seq0;
    P.draws = a.draws;
    P.tokens = a.tokens;
    if (!P.u && !P.draws && a.mode != Q35_SAMPLE_GREEDY)
        return set_error(Q35_ERR_INVALID, "sampling: neither uniforms nor draw counters");
    const size_t smem = sizeof(float) * (size_t)pidx(a.V);
    static bool attr_set[64] = {};
    int dev = 0;
    Q35_CUDA_TRY(cudaGetDevice(&dev));
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        Q35_CUDA_TRY(cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)(sizeof(float) * (size_t)pidx(SMAXV))));
        attr_set[dev] = true;
    }
    sample_kernel<<<a.rows, SNT, smem, s>>>(P);
    Q35_CUDA_TRY(cudaGetLastError());
    return Q35_OK;
}

}  // namespace q35

using namespace q35;

namespace {

// host drop-ins: one row of host logits, the draw u given
int sample_host(q35_ctx ctx, int mode, const float *logits, int32_t vocab, float temperature, int32_t k, float p,
                float u, int32_t *token) {
    if (!logits || !token) return set_error(Q35_ERR_INVALID, "NULL argument");
    int st = sample_check(mode, vocab);
    if (st) return st;
    if (!ctx) {
        st = default_ctx(&ctx);
        if (st) return st;
    }
    if (!(u >= 0.0f && u < 1.0f)) return set_error(Q35_ERR_INVALID, "sampling: u must lie in [0,1)");
    DeviceGuard g(ctx->device);
    std::lock_guard<std::mutex> lk(ctx->mu);
    const size_t lb = round_up(sizeof(float) * (size_t)vocab, 256);
    st = ensure_scratch(ctx, lb + 256, lb + 256);
    if (st) return st;
    char *d = static_cast<char *>(ctx->d_scratch);
    char *h = static_cast<char *>(ctx->h_pinned);
    std::memcpy(h, logits, sizeof(float) * (size_t)vocab);
    std::memcpy(h + lb, &u, sizeof(float));
    cudaStream_t s = ctx->stream;
    Q35_CUDA_TRY(cudaMemcpyAsync(d, h, lb + sizeof(float), cudaMemcpyHostToDevice, s));
    SampleRows a;
    a.logits = reinterpret_cast<const float *>(d);
    a.Vl = vocab;
    a.Rtot = 1;
    a.V = vocab;
    a.row0 = 0;
    a.rows = 1;
    a.mode = mode;
    a.temperature = temperature;
    a.top_k = k;
    a.top_p = p;
    a.u = reinterpret_cast<const float *>(d + lb);
    a.tokens = reinterpret_cast<int32_t *>(d + lb + 128);
    st = launch_sample(a, s);
    if (st) return st;
    Q35_CUDA_TRY(cudaMemcpyAsync(h + lb + 128, d + lb + 128, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    Q35_CUDA_TRY(cudaStreamSynchronize(s));
    std::memcpy(token, h + lb + 128, sizeof(int32_t));
    return Q35_OK;
}

}  // namespace

extern "C" {

int q35_sample_greedy(q35_ctx ctx, const float *logits, int32_t vocab, int32_t *token) {
    return sample_host(ctx, Q35_SAMPLE_GREEDY, logits, vocab, 0.0f, 0, 0.0f, 0.0f, token);
}

int q35_sample_temperature(q35_ctx ctx, const float *logits, int32_t vocab, float temperature, float u,
                           int32_t *token) {
    return sample_host(ctx, Q35_SAMPLE_TEMPERATURE, logits, vocab, temperature, 0, 0.0f, u, token);
}

int q35_sample_top_k(q35_ctx ctx, const float *logits, int32_t vocab, int32_t k, float u, int32_t *token) {
    return sample_host(ctx, Q35_SAMPLE_TOP_K, logits, vocab, 0.0f, k, 0.0f, u, token);
}

int q35_sample_top_p(q35_ctx ctx, const float *logits, int32_t vocab, float p, float u, int32_t *token) {
    return sample_host(ctx, Q35_SAMPLE_TOP_P, logits, vocab, 0.0f, 0, p, u, token);
}

int q35_sample_dev(q35_ctx ctx, int32_t mode, const float *logits, int32_t rows, int32_t vocab, float temperature,
                   int32_t top_k, float top_p, const float *u, int32_t *tokens) {
    if (!ctx || !logits || !tokens || (mode != Q35_SAMPLE_GREEDY && !u))
        return set_error(Q35_ERR_INVALID, "NULL argument");
    if (rows < 0) return set_error(Q35_ERR_INVALID, "sampling: negative row count");
    DeviceGuard g(ctx->device);
    SampleRows a;
    a.logits = logits;
    a.Vl = vocab;
    a.Rtot = rows;
    a.V = vocab;
    a.row0 = 0;
    a.rows = rows;
    a.mode = mode;
    a.temperature = temperature;
    a.top_k = top_k;
    a.top_p = top_p;
    a.u = u;
    a.tokens = tokens;
    return launch_sample(a, ctx->stream);
}

}  // extern "C"
