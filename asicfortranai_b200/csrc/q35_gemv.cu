// q35_gemv.cu -- decode GEMV / skinny GEMM on CUDA cores (dp4a), exact int32.
//
// Computes, for the reference kernels matmul_3p5bit_awq (matmul_3p5bit_dynamic.f90:42-64)
// and matmul_int4_awq (matmul_int4_groq.f90:117-137):
//   C(i,j) = sum_k A(i,k) * code(k,j)          (int32, exact)
//   y(i,j) = (float(C) + offset_j) * scale_j   (3.5-bit, :80)   or  float(C) * scale_j (INT4)
//
// Three launch shapes.  Per column group (when all column groups fit on the GPU at once):
// CTA b takes column group b, its warps split the k-blocks and add their exact partial
// sums in shared memory.  The same split over a thread-block cluster when few column
// groups leave SMs idle (below).  Stream (larger N): the grid holds as many CTAs as fit on
// the GPU at once; the (column group, k-block) tiles, stored column-group major, are cut
// into one contiguous range per warp of equal length, so every warp streams the same
// number of bytes and no wave tail is left.  A warp walks its range through a private ring
// of shared-memory stages; lane 0 fills each stage with one TMA bulk copy (cp.async.bulk,
// a whole 3.5 KB / 4 KB tile, completion counted on an mbarrier), so several tiles per
// warp are in flight without occupying registers or per-thread request slots.  Each lane
// owns one output column.  Launched with programmatic dependent launch: a CTA initialises
// its barriers and starts its weight stream (the first tile of each warp) before waiting
// (griddepcontrol.wait) for the kernel ahead of it.  Every mbarrier wait is bounded: when
// it gives up the kernel records Q35_ERR_TIMEOUT in the workspace error word, drains its
// own copies (again bounded) and leaves.
//
// Right after the wait the CTA stages its activation rows for the k-blocks it consumes
// (the whole K but in the split per-group form): with 16-byte aligned rows and K a
// multiple of 16, one bulk copy per row into shared memory, issued before the rest of the
// weight ring (an SM's copies complete about in issue order, and every warp needs the
// activations first), then turned in place into the even/odd image order; otherwise
// 8-byte loads.  Beside the image, the per-k-block bias corrections (codes are stored
// biased, so sum a*code = sum a*biased - sum a*bias, see q35_internal.cuh).
//
// Per-group form split over a cluster (few column groups): the S CTAs of a thread-block
// cluster share one column group, CTA c taking k-blocks [KB*c/S, KB*(c+1)/S); each CTA
// adds its warps' sums in shared memory, stores the total into slot c of CTA 0's shared
// memory (st.shared::cluster), and after a cluster barrier CTA 0 adds the S slots and
// runs the epilogue.  The barrier's first half (arrive at the start of a row chunk, wait
// before the remote stores) guarantees every CTA of the cluster is running.
//
// Multiply without shifts: a weight field is masked in place and multiplied with
// dp4a.u32.s32, which yields 2^s times the wanted partial sum; partial sums of equal
// scale 2^s share an accumulator, and the accumulators are combined with exact
// arithmetic right shifts at the end (every term of accumulator s is a multiple of 2^s).
// 3.5-bit costs 21 masks + 21 dp4a per 64 weights, INT4 2 + 2 per 8 weights.
//
// Stream shape: a run of k-blocks of one column group inside a warp's range is a segment.  A segment
// that covers the whole K writes its outputs directly; otherwise (only a warp's first
// and last segment can be partial) it adds its exact partial sums into an int32
// workspace at once (atomicAdd: integer addition is order free, so the result is
// bit-identical to a single pass) and, after the warp's stream has ended, adds its
// k-block count to the column group's counter with release/acquire semantics; the
// segment that completes the count reads the totals back with atomicExch(.., 0),
// leaving the workspace zero for the next call, runs the dequant epilogue and resets
// the counter.
#include <algorithm>

#include "q35_expf.h"
#include "q35_internal.cuh"

#ifndef Q35_GEMV_PF
#define Q35_GEMV_PF 0   // tiles prefetched into L2 beyond the shared-memory ring
#endif

namespace q35 {

constexpr int GEMV_WARPS = 8;
constexpr int GEMV_THREADS = GEMV_WARPS * 32;
constexpr int GEMV_MT_MAX = 4;      // activation rows per pass
constexpr int GEMV_MAX_K = 131072;  // keeps every scale accumulator below 2^31

struct GemvParams {
    const uint4 *tiles;
    const float *scales, *offsets;
    int32_t KB, CG, N, K;
    const int8_t *x;
    int64_t sx_row, sx_k;
    int32_t M;
    int32_t *C;
    float *y;
    int64_t so_row, so_col;
    int32_t *ws_acc;         // [M][CG*32], zero between calls
    uint32_t *counters;      // [row chunks][CG], zero between calls
    int vec_x;               // activations can be read 8 bytes at a time
    int bulk_x;              // rows 16-byte aligned, K a multiple of 16: one bulk copy per row
    int per_group;           // one CTA per column group, K split over its warps (no workspace)
    int split;               // per-group form: CTAs of a cluster sharing one column group's K
    int8_t *sq;              // SwiGLU output [M][N/2] int8 (interleaved gate/up columns), or null
    int *err;                // device error word (Q35_ERR_TIMEOUT on a failed wait)
    const float *res;        // optional residual: y = res + dequant(C), same strides as y
    int has_rope;            // q|k|v epilogue (rope): RoPE, q out, K and V into the cache
    GemvRope rope;
};

__device__ __forceinline__ int dp4au(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred P1;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2;\n\t"
                 "selp.b32 %0, 1, 0, P1;\n\t}"
                 : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
// bounded wait on one phase of an mbarrier
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    for (uint32_t i = 0; i < (1u << 26); ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}
__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}
// counter update that publishes this warp's partial sums (release) and, for the warp
// that completes the count, makes every other warp's partial sums visible (acquire)
__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned *p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// thread-block cluster barrier (release on arrive, acquire on wait) and a store into the
// shared memory of another CTA of the cluster
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait;" ::: "memory"); }
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void st_cluster_s32(uint32_t local_addr, uint32_t cta, int v) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(cta));
    asm volatile("st.shared::cluster.s32 [%0], %1;" ::"r"(remote), "r"(v) : "memory");
}

// 3.5-bit: accumulators a[0..5] hold partial sums scaled by 1, 8, 16, 32, 64, 128.
// Per group of 32 pairs (7 words): the odd code (bits 0..2) meets the odd activations
// at scale 1, the even code (bits 3..6) the even activations at scale 8, and bit 7 of
// word i, bit i of a stuffed pair's field, meets the stuffed pairs' odd (i < 3) or even
// (i >= 3) activations at scale 128 / 2^i or 128 / 2^(i-3).
__device__ __forceinline__ void dot35(const uint32_t (&W)[32], const uint32_t *img, int (&a)[7]) {
    const uint4 *E4 = reinterpret_cast<const uint4 *>(img);
    const uint4 *O4 = reinterpret_cast<const uint4 *>(img + 32);
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        const uint4 e0 = E4[2 * g], e1 = E4[2 * g + 1];
        const uint4 o0 = O4[2 * g], o1 = O4[2 * g + 1];
        const uint32_t E[8] = {e0.x, e0.y, e0.z, e0.w, e1.x, e1.y, e1.z, e1.w};
        const uint32_t O[8] = {o0.x, o0.y, o0.z, o0.w, o1.x, o1.y, o1.z, o1.w};
#pragma unroll
        for (int i = 0; i < 7; ++i) {
            const uint32_t w = W[7 * g + i];
            a[0] = dp4au(w & 0x07070707u, O[i], a[0]);
            a[1] = dp4au(w & 0x78787878u, E[i], a[1]);
            const uint32_t m = w & 0x80808080u;
            // scale slot of bit i: 128,64,32 (odd field bits), 128,64,32,16 (even field bits)
            constexpr int slot[7] = {5, 4, 3, 5, 4, 3, 2};
            a[slot[i]] = dp4au(m, i < 3 ? O[7] : E[7], a[slot[i]]);
        }
    }
}

__device__ __forceinline__ void dot4(const uint32_t (&W)[32], const uint32_t *img, int (&a)[7]) {
    const uint4 *I4 = reinterpret_cast<const uint4 *>(img);
#pragma unroll
    for (int q = 0; q < 16; ++q) {
        const uint4 e = I4[q];
        const uint32_t w0 = W[2 * q], w1 = W[2 * q + 1];
        a[0] = dp4au(w0 & 0x0F0F0F0Fu, e.x, a[0]);
        a[4] = dp4au(w0 & 0xF0F0F0F0u, e.y, a[4]);
        a[1] = dp4au(w1 & 0x0F0F0F0Fu, e.z, a[1]);   // a[1] used at scale 1 here
        a[5] = dp4au(w1 & 0xF0F0F0F0u, e.w, a[5]);   // a[5] used at scale 16 here
    }
}

__device__ __forceinline__ int combine(int FMT, const int (&a)[7]) {
    if (FMT == Q35_FMT_3P5BIT)
        return a[0] + (a[1] >> 3) + (a[2] >> 4) + (a[3] >> 5) + (a[4] >> 6) + (a[5] >> 7);
    return a[0] + a[1] + (a[4] >> 4) + (a[5] >> 4);
}

// a column's scale and offset, loaded ahead of the epilogue (the weights' side of the
// dequant: nothing the previous kernel writes)
struct ColQ {
    float sc = 0.0f, of = 0.0f;
};
__device__ __forceinline__ ColQ colq(const GemvParams &p, int64_t j, bool valid) {
    ColQ q;
    if (valid) {
        q.sc = p.scales[j];
        if (p.offsets) q.of = p.offsets[j];
    }
    return q;
}

__device__ __forceinline__ float dequant(int FMT, int32_t c, ColQ q) {
    float f = __int2float_rn(c);
    if (FMT == Q35_FMT_3P5BIT) return __fmul_rn(__fadd_rn(f, q.of), q.sc);
    return __fmul_rn(f, q.sc);
}

// epilogue store of one output: C, and y = dequant (+ residual, the layer's x + f(x),
// transformer_layer.f90:550 and :557)
template <int FMT>
__device__ __forceinline__ void store_out(const GemvParams &p, int row, int64_t j, int32_t c, ColQ q) {
    const int64_t o = row * p.so_row + j * p.so_col;
    if (p.C) p.C[o] = c;
    if (p.y) {
        float v = dequant(FMT, c, q);
        if (p.res) v = __fadd_rn(p.res[o], v);
        p.y[o] = v;
    }
}

// one row's outputs of a warp's 32 columns (j = this lane's column, valid = j < N, q its
// scale and offset); every lane of the warp calls it.  With sq set the columns are (gate,
// up) pairs: the even lane forms silu(gate) * up (swiglu_kernel, transformer_layer.f90:
// 212-229) and its int8 value.
// the q|k|v epilogue (rope_kv_kernel's arithmetic, transformer_layer.f90:183-205 and
// :322-329): each lane rotates its own element of the pair (2d, 2d+1), the partner's value
// arriving by shuffle; v columns go to the cache unrotated.  Every lane of the warp calls it.
template <int FMT>
__device__ __forceinline__ void store_rope(const GemvParams &p, int row, int64_t j, int32_t c, bool valid, ColQ q) {
    const GemvRope &g = p.rope;
    const float v = valid ? dequant(FMT, c, q) : 0.0f;
    const float u = __shfl_xor_sync(0xffffffffu, v, 1);
    if (!valid) return;
    if (p.y) p.y[row * p.so_row + j * p.so_col] = v;
    const int r = g.row0 + row;
    const int s = g.row_seq[r], i = g.row_i[r];
    const int pos = g.cache_pos[s] + i;
    if (pos < 0 || pos >= g.max_seq) {
        atomicExch(p.err, Q35_ERR_INVALID);
        return;
    }
    const int QN = g.H * g.D, KN = g.KVH * g.D;
    const int jj = (int)j;
    const bool isq = jj < QN, isv = jj >= QN + KN;
    const int col = isq ? jj : (isv ? jj - QN - KN : jj - QN);
    const int hh = col / g.D, dd = col - hh * g.D;
    const size_t co = ((((size_t)s * g.n_layers + g.layer) * g.KVH + hh) * g.max_seq + pos) * g.D + dd;
    if (isv) {
        g.vc[co] = v;
        return;
    }
    const float2 cs = g.cs[(size_t)(g.rope_mode ? pos : i) * (g.D / 2) + (dd >> 1)];
    const bool odd = dd & 1;
    const float a = odd ? u : v, b = odd ? v : u;
    const float o = odd ? __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x))
                        : __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
    if (isq) g.q[(size_t)r * QN + col] = o;
    else g.kc[co] = o;
}

template <int FMT>
__device__ __forceinline__ void store_row(const GemvParams &p, int row, int64_t j, int32_t c, bool valid, ColQ q) {
    if (p.has_rope) {
        store_rope<FMT>(p, row, j, c, valid, q);
    } else if (p.sq) {
        const float v = valid ? dequant(FMT, c, q) : 0.0f;
        const float up = __shfl_xor_sync(0xffffffffu, v, 1);
        if (valid && (j & 1) == 0) {
            const float sw = __fdiv_rn(v, __fadd_rn(1.0f, q35_expf(-v)));
            p.sq[(int64_t)row * (p.N / 2) + (j >> 1)] = quant127(__fmul_rn(sw, up));
        }
    } else if (valid) {
        store_out<FMT>(p, row, j, c, q);
    }
}

template <int FMT>
struct Tile {
    static constexpr int NC = (FMT == Q35_FMT_3P5BIT) ? 7 : 8;    // 16-byte chunks per lane
    static constexpr int BYTES = NC * 512;
    static constexpr int U4 = NC * 32;
};

// two CTAs per SM for the one-row forms and the 3.5-bit two-row form (at most 128
// registers a thread)
template <int FMT, int MT, int D>
__global__ void __launch_bounds__(GEMV_THREADS, (MT == 1 || (FMT == Q35_FMT_3P5BIT && MT == 2)) ? 2 : 1)
gemv_kernel(const GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    using T = Tile<FMT>;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int KB = p.KB;
    // per-group form: column group cgb, and with a cluster split (S > 1) this CTA's share
    // [kb0, kb0 + KBw) of its k-blocks; the stream form sees every k-block
    const int S = p.per_group ? p.split : 1;
    const int crank = S > 1 ? (int)cluster_ctarank() : 0;
    const int64_t cgb = S > 1 ? (int64_t)cluster_id_x() : (int64_t)blockIdx.x;
    const int kb0 = p.per_group ? (int)((int64_t)KB * crank / S) : 0;
    const int KBw = p.per_group ? (int)((int64_t)KB * (crank + 1) / S) - kb0 : KB;
    // KBl: the image capacity, the largest share, the same in every CTA of a cluster so
    // that the areas below sit at the same offsets in all of them (CTA 0's slots are
    // addressed through the other CTAs' own layout)
    const int KBl = p.per_group ? (int)ceil_div(KB, S) : KB;
    // layout: [ring: warps x D tiles][img: MT x KBl x 256 B][corr: MT x KBl int][mbarriers]
    //         [red: warps x MT x 32 int, per-group form][cl: S x MT x 32 int, cluster split]
    uint8_t *ring = smem + (size_t)warp * D * T::BYTES;
    uint32_t *img = reinterpret_cast<uint32_t *>(smem + (size_t)GEMV_WARPS * D * T::BYTES);
    int32_t *corr = reinterpret_cast<int32_t *>(reinterpret_cast<uint8_t *>(img) + (size_t)MT * KBl * KBLK);
    const uint32_t bars0 = (uint32_t)__cvta_generic_to_shared(
        reinterpret_cast<uint8_t *>(corr) + round_up((int64_t)MT * KBl * 4, 8));
    const uint32_t bars = bars0 + warp * D * 8;
    const uint32_t xbar = bars0 + GEMV_WARPS * D * 8;   // the activation copy's barrier
    int32_t *red = reinterpret_cast<int32_t *>(reinterpret_cast<uint8_t *>(corr) + round_up((int64_t)MT * KBl * 4, 8) +
                                               GEMV_WARPS * D * 8 + 16);
    int32_t *cl = red + GEMV_WARPS * MT * 32;
    const uint32_t ring_s = (uint32_t)__cvta_generic_to_shared(ring);
    const uint8_t *gtiles = reinterpret_cast<const uint8_t *>(p.tiles);

    const int64_t U = (int64_t)p.CG * KB;
    const int64_t Wt = (int64_t)gridDim.x * GEMV_WARPS;
    const int64_t gw = (int64_t)blockIdx.x * GEMV_WARPS + warp;
    // stream mode: one balanced range of tiles per warp across the grid; per-group mode:
    // the CTA takes column group cgb (its k-block share) and its warps split the k-blocks
    const int64_t u0 = p.per_group ? cgb * KB + kb0 + (int64_t)KBw * warp / GEMV_WARPS : U * gw / Wt;
    const int64_t u1 = p.per_group ? cgb * KB + kb0 + (int64_t)KBw * (warp + 1) / GEMV_WARPS : U * (gw + 1) / Wt;
    const int64_t Np = (int64_t)p.CG * 32;
    const int nchunks = (p.M + MT - 1) / MT;

    if (lane == 0) {
        for (int s = 0; s < D; ++s) mbar_init(bars + 8 * s, 1);
        if (tid == 0) mbar_init(xbar, 1);
        mbar_fence_init();
    }
    __syncthreads();
    // programmatic dependent launch: let the next kernel in the stream begin its own
    // weight stream as our CTAs retire
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    uint32_t phase = 0;       // bit s: parity of the next completion of stage s
    uint32_t xphase = 0;      // parity of the activation barrier's next completion
    bool failed = false;
    // per-group form: this lane's column and its scale/offset, loaded before the wait on
    // the previous kernel (weights do not depend on it)
    const ColQ gq = p.per_group ? colq(p, cgb * 32 + lane, cgb * 32 + lane < p.N) : ColQ();

    for (int chunk = 0; chunk < nchunks; ++chunk) {
        const int r0 = chunk * MT;
        // cluster split: the first half of this row chunk's cluster barrier (its wait, before
        // the partial sums are stored into CTA 0, ensures every CTA of the cluster has
        // started and that CTA 0 has read the previous chunk's sums)
        if (S > 1) cluster_arrive();
        // ---- before the wait: only the first tile of this warp's range (every copy issued
        // here, L2 prefetches included, would complete ahead of the activation copy) ----
        if (lane == 0 && !failed && u0 < u1) {
            mbar_expect_tx(bars, T::BYTES);
            bulk_g2s(ring_s, gtiles + (size_t)u0 * T::BYTES, T::BYTES, bars);
        }
        // weights never depend on the previous kernel; activations, the workspace and the
        // outputs may: wait for the predecessor grid here (a no-op without one)
        if (chunk == 0) asm volatile("griddepcontrol.wait;" ::: "memory");
        // ---- stage the activation image of rows r0.., this CTA's k-blocks, and corrections ----
        // The activation copy is issued before the rest of the ring's tiles: the SM's copies
        // complete about in issue order, and the image is what every warp needs first
        const int64_t kbeg = (int64_t)kb0 * KBLK;
        const uint32_t nrow = (uint32_t)min((int64_t)KBw * KBLK, (int64_t)p.K - kbeg);
        if (p.bulk_x && tid == 0) {
            if (chunk > 0) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            uint32_t total = 0;
            for (int r = 0; r < MT; ++r)
                if (r0 + r < p.M) total += nrow;
            mbar_expect_tx(xbar, total);
            for (int r = 0; r < MT; ++r)
                if (r0 + r < p.M)
                    bulk_g2s((uint32_t)__cvta_generic_to_shared(img + (size_t)r * KBl * 64),
                             p.x + (int64_t)(r0 + r) * p.sx_row + kbeg, nrow, xbar);
        }
        if (p.bulk_x) __syncthreads();   // the activation copy first, then the ring's other tiles
        if (lane == 0 && !failed) {
            for (int s = 1; s < D && u0 + s < u1; ++s) {
                mbar_expect_tx(bars + 8 * s, T::BYTES);
                bulk_g2s(ring_s + s * T::BYTES, gtiles + (size_t)(u0 + s) * T::BYTES, T::BYTES, bars + 8 * s);
            }
            for (int s = D; s < D + Q35_GEMV_PF && u0 + s < u1; ++s)
                bulk_prefetch_l2(gtiles + (size_t)(u0 + s) * T::BYTES, T::BYTES);
        }
        if (p.bulk_x) {
            // each row's window arrived by one bulk copy; each warp turns its k-blocks into
            // the even/odd image in place (reads, __syncwarp, writes)
            if (!mbar_wait(xbar, xphase)) {
                failed = true;
                if (tid == 0) atomicExch(p.err, Q35_ERR_TIMEOUT);
            }
            xphase ^= 1u;
            for (int t = warp; t < MT * KBw; t += GEMV_WARPS) {
                const int r = t / KBw, kb = t % KBw;
                uint32_t *im = img + ((size_t)r * KBl + kb) * 64;
                const int64_t kv = (int64_t)p.K - kbeg - (int64_t)kb * KBLK;   // valid k of this block
                uint32_t lo = im[2 * lane], hi = im[2 * lane + 1];
                if (r0 + r >= p.M || 8 * lane >= kv || failed) lo = hi = 0u;
                __syncwarp();
                const uint32_t e = __byte_perm(lo, hi, 0x6420);
                const uint32_t o = __byte_perm(lo, hi, 0x7531);
                im[lane] = e;
                im[32 + lane] = o;
                int c = (FMT == Q35_FMT_3P5BIT) ? __dp4a((int)e, 0x08080808, __dp4a((int)o, 0x04040404, 0))
                                                : __dp4a((int)e, 0x08080808, __dp4a((int)o, 0x08080808, 0));
#pragma unroll
                for (int s = 16; s > 0; s >>= 1) c += __shfl_xor_sync(0xffffffffu, c, s);
                if (lane == 0) corr[r * KBl + kb] = c;
            }
        }
        // (other layouts: loads of up to 8 items per warp are issued before any is used)
        for (int t0 = warp; !p.bulk_x && t0 < MT * KBw; t0 += 8 * GEMV_WARPS) {
            uint32_t lo[8], hi[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int t = t0 + i * GEMV_WARPS;
                lo[i] = 0;
                hi[i] = 0;
                if (t >= MT * KBw) continue;
                const int r = t / KBw, kb = kb0 + t % KBw, row = r0 + r;
                const int64_t k0 = (int64_t)kb * KBLK + 8 * lane;   // 8 consecutive k per lane
                if (row >= p.M) continue;
                const int8_t *xr = p.x + row * p.sx_row;
                if (p.vec_x && k0 + 8 <= p.K) {
                    const uint2 v = *reinterpret_cast<const uint2 *>(xr + k0);
                    lo[i] = v.x;
                    hi[i] = v.y;
                } else {
#pragma unroll
                    for (int b = 0; b < 8; ++b) {
                        const int64_t k = k0 + b;
                        const uint32_t v = (k < p.K) ? (uint8_t)xr[k * p.sx_k] : 0u;
                        if (b < 4) lo[i] |= v << (8 * b); else hi[i] |= v << (8 * (b - 4));
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int t = t0 + i * GEMV_WARPS;
                if (t >= MT * KBw) break;
                const int r = t / KBw, kb = t % KBw;   // kb: index within the window
                const uint32_t e = __byte_perm(lo[i], hi[i], 0x6420);   // k0, k0+2, k0+4, k0+6
                const uint32_t o = __byte_perm(lo[i], hi[i], 0x7531);   // k0+1, k0+3, k0+5, k0+7
                uint32_t *im = img + ((size_t)r * KBl + kb) * 64;
                im[lane] = e;
                im[32 + lane] = o;
                int c = (FMT == Q35_FMT_3P5BIT) ? __dp4a((int)e, 0x08080808, __dp4a((int)o, 0x04040404, 0))
                                                : __dp4a((int)e, 0x08080808, __dp4a((int)o, 0x08080808, 0));
#pragma unroll
                for (int s = 16; s > 0; s >>= 1) c += __shfl_xor_sync(0xffffffffu, c, s);
                if (lane == 0) corr[r * KBl + kb] = c;
            }
        }
        __syncthreads();

        if (u0 < u1 && !failed) {
            // the image and corrections indexed by the column group's k-block number
            const uint32_t *imgk = img - (size_t)kb0 * 64;
            const int32_t *corrk = corr - kb0;
            int acc[MT][7];
            int csum[MT];
#pragma unroll
            for (int r = 0; r < MT; ++r) {
                csum[r] = 0;
#pragma unroll
                for (int s = 0; s < 7; ++s) acc[r][s] = 0;
            }
            int64_t cg = u0 / KB;
            int kb = (int)(u0 - cg * KB);
            int64_t pend_cg[2] = {0, 0};
            int pend_kb[2] = {0, 0};
            ColQ pend_q[2];
            // stream form: the scale/offset of the segment's column group, loaded as the
            // segment starts so that its latency hides behind the segment's tiles
            ColQ segq = p.per_group ? gq : colq(p, cg * 32 + lane, cg * 32 + lane < p.N);
            int npend = 0;
            int seg_kb = 0;
            int stage = 0;
            const int n_units = (int)(u1 - u0);
            for (int it = 0; it < n_units; ++it) {
                const uint32_t bar = bars + 8 * stage;
                if (!mbar_wait(bar, (phase >> stage) & 1u)) {
                    failed = true;
                    if (lane == 0) atomicExch(p.err, Q35_ERR_TIMEOUT);
                    // drain this warp's other copies in flight (bounded), then stop
                    for (int v = it + 1; v < n_units && v < it + D; ++v) {
                        const int sv = v % D;
                        mbar_wait(bars + 8 * sv, (phase >> sv) & 1u);
                    }
                    break;
                }
                phase ^= 1u << stage;
                uint32_t W[32];
                const uint4 *sp = reinterpret_cast<const uint4 *>(ring + stage * T::BYTES + lane * 16);
#pragma unroll
                for (int c = 0; c < T::NC; ++c) {
                    const uint4 v = sp[c * 32];
                    W[4 * c] = v.x; W[4 * c + 1] = v.y; W[4 * c + 2] = v.z; W[4 * c + 3] = v.w;
                }
#pragma unroll
                for (int r = 0; r < MT; ++r) {
                    const uint32_t *im = imgk + ((size_t)r * KBl + kb) * 64;
                    if (FMT == Q35_FMT_3P5BIT) dot35(W, im, acc[r]); else dot4(W, im, acc[r]);
                    csum[r] += corrk[r * KBl + kb];
                }
                // every lane has consumed its words of this stage: refill it with the tile
                // D ahead (the stage's shared-memory reads are complete, their values used)
                __syncwarp();
                if (lane == 0 && it + D < n_units) {
                    mbar_expect_tx(bar, T::BYTES);
                    bulk_g2s(ring_s + stage * T::BYTES, gtiles + (size_t)(u0 + it + D) * T::BYTES, T::BYTES, bar);
                }
                if (Q35_GEMV_PF > 0 && lane == 0 && it + D + Q35_GEMV_PF < n_units)
                    bulk_prefetch_l2(gtiles + (size_t)(u0 + it + D + Q35_GEMV_PF) * T::BYTES, T::BYTES);
                ++seg_kb;
                ++kb;
                stage = (stage + 1 == D) ? 0 : stage + 1;

                if (it + 1 == n_units || kb == KB) {
                    // ---- segment end: column group cg, seg_kb k-blocks ----
                    const int64_t j = cg * 32 + lane;
                    int tot[MT];
#pragma unroll
                    for (int r = 0; r < MT; ++r) tot[r] = combine(FMT, acc[r]) - csum[r];
                    if (p.per_group) {
                        // the CTA's warps meet in shared memory (below)
#pragma unroll
                        for (int r = 0; r < MT; ++r) red[(warp * MT + r) * 32 + lane] = tot[r];
                    } else if (seg_kb == KB) {
#pragma unroll
                        for (int r = 0; r < MT; ++r) {
                            const int row = r0 + r;
                            if (row < p.M) store_row<FMT>(p, row, j, tot[r], j < p.N, segq);
                        }
                    } else {
                        // partial segment (at most two per warp: its first and its last):
                        // post the exact partial sums now, settle the counter after the
                        // stream so no memory fence waits on copies still in flight
                        if (j < p.N) {
#pragma unroll
                            for (int r = 0; r < MT; ++r)
                                if (r0 + r < p.M && tot[r] != 0) atomicAdd(&p.ws_acc[(r0 + r) * Np + j], tot[r]);
                        }
                        if (npend < 2) {   // only a warp's first and last segment can be partial
                            pend_cg[npend] = cg;
                            pend_kb[npend] = seg_kb;
                            pend_q[npend] = segq;
                            ++npend;
                        } else if (lane == 0) {
                            atomicExch(p.err, Q35_ERR_STATE);
                        }
                    }
#pragma unroll
                    for (int r = 0; r < MT; ++r) {
                        csum[r] = 0;
#pragma unroll
                        for (int s = 0; s < 7; ++s) acc[r][s] = 0;
                    }
                    seg_kb = 0;
                    kb = 0;
                    ++cg;
                    if (!p.per_group && it + 1 < n_units) segq = colq(p, cg * 32 + lane, cg * 32 + lane < p.N);
                }
            }
            // ---- settle the partial segments: the warp completing a column group's
            // k-block count reads the totals back and runs the epilogue ----
            __syncwarp();   // orders the lanes' adds before lane 0's release
            for (int q = 0; q < npend; ++q) {
                unsigned last = 0;
                if (lane == 0) {
                    unsigned *ctr = &p.counters[(size_t)chunk * p.CG + pend_cg[q]];
                    last = (atom_add_acq_rel(ctr, (unsigned)pend_kb[q]) + (unsigned)pend_kb[q] == (unsigned)KB);
                }
                last = __shfl_sync(0xffffffffu, last, 0);
                __syncwarp();
                if (last) {
                    const int64_t j = pend_cg[q] * 32 + lane;
#pragma unroll
                    for (int r = 0; r < MT; ++r) {
                        const int row = r0 + r;
                        if (row < p.M)
                            store_row<FMT>(p, row, j, j < p.N ? atomicExch(&p.ws_acc[row * Np + j], 0) : 0, j < p.N,
                                           pend_q[q]);
                    }
                    if (lane == 0) p.counters[(size_t)chunk * p.CG + pend_cg[q]] = 0u;
                }
            }
        }
        if (p.per_group) {
            // warps without k-blocks add nothing; then the sum over warps (integer, exact)
            if (u0 == u1 || failed)
                for (int r = 0; r < MT; ++r) red[(warp * MT + r) * 32 + lane] = 0;
            __syncthreads();
            const int64_t j = cgb * 32 + lane;
            if (S == 1) {
                for (int r = warp; r < MT; r += GEMV_WARPS) {
                    int t = 0;
#pragma unroll
                    for (int w2 = 0; w2 < GEMV_WARPS; ++w2) t += red[(w2 * MT + r) * 32 + lane];
                    const int row = r0 + r;
                    if (row < p.M) store_row<FMT>(p, row, j, t, j < p.N, gq);
                }
            } else {
                // cluster split: each CTA's sums go into slot crank of CTA 0's area; after
                // the barrier CTA 0 adds the S slots (integer, exact) and stores
                cluster_wait();
                for (int r = warp; r < MT; r += GEMV_WARPS) {
                    int t = 0;
#pragma unroll
                    for (int w2 = 0; w2 < GEMV_WARPS; ++w2) t += red[(w2 * MT + r) * 32 + lane];
                    st_cluster_s32((uint32_t)__cvta_generic_to_shared(cl + (crank * MT + r) * 32 + lane), 0u, t);
                }
                cluster_arrive();
                cluster_wait();
                if (crank == 0) {
                    for (int r = warp; r < MT; r += GEMV_WARPS) {
                        int t = 0;
                        for (int c = 0; c < S; ++c) t += cl[(c * MT + r) * 32 + lane];
                        const int row = r0 + r;
                        if (row < p.M) store_row<FMT>(p, row, j, t, j < p.N, gq);
                    }
                }
            }
        }
        __syncthreads();   // the image (and the reduction area) is rewritten by the next row chunk
    }
}

static int sm_count(int dev) {
    static int cached[64] = {0};
    if (dev < 0 || dev >= 64) return 148;
    if (!cached[dev]) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
        cached[dev] = v;
    }
    return cached[dev];
}

static int pick_mt(int32_t M) { return M <= 1 ? 1 : (M <= 2 ? 2 : 4); }

static size_t smem_bytes(int fmt, int MT, int D, int KB, int S = 1);

// rows per pass: pick_mt, unless the activation image of that many rows over a long K
// does not fit in shared memory; then fewer rows per pass (more passes), as long as the
// passes still fit the row-chunk counters of the workspace (64 / GEMV_MT_MAX of them)
static int fit_mt(const Weights &w, int32_t M) {
    static int optin_cache[64] = {0};
    int optin = 0;
    if (w.device >= 0 && w.device < 64 && optin_cache[w.device]) {
        optin = optin_cache[w.device];
    } else {
        if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, w.device) != cudaSuccess) optin = 0;
        if (optin > 0 && w.device >= 0 && w.device < 64) optin_cache[w.device] = optin;
    }
    int mt = pick_mt(M);
    while (optin > 0 && mt > 1 && smem_bytes(w.format, mt, 2, w.KB) > (size_t)optin &&
           ceil_div((int64_t)M, (int64_t)(mt / 2)) <= 64 / GEMV_MT_MAX)
        mt /= 2;
    return mt;
}

// KB: the k-blocks whose activation image a CTA stages; S: CTAs of a cluster split
static size_t smem_bytes(int fmt, int MT, int D, int KB, int S) {
    const size_t tb = fmt == Q35_FMT_3P5BIT ? Tile<Q35_FMT_3P5BIT>::BYTES : Tile<Q35_FMT_INT4>::BYTES;
    return (size_t)GEMV_WARPS * D * tb + (size_t)MT * KB * KBLK + round_up((int64_t)MT * KB * 4, 8) +
           (size_t)GEMV_WARPS * D * 8 + 16 + (size_t)GEMV_WARPS * MT * 32 * 4 + (S > 1 ? (size_t)S * MT * 32 * 4 : 0);
}

size_t gemv_workspace_acc_elems(const Weights &w, int32_t M) { return (size_t)M * w.CG * 32; }

size_t gemv_workspace_tickets(const Weights &w) {
    return (size_t)w.CG * ((64 + GEMV_MT_MAX - 1) / GEMV_MT_MAX);
}

// shared-memory size and CTAs per SM of gemv_kernel<FMT, MT, D> for K-blocks KB (the
// dynamic shared-memory limit raised once per device, occupancies cached)
template <int FMT, int MT, int D>
static int occupancy(const Weights &w, size_t &smem, int &per_sm, int KBw = -1, int S = 1) {
    auto kern = gemv_kernel<FMT, MT, D>;
    smem = smem_bytes(FMT, MT, D, KBw < 0 ? w.KB : KBw, S);
    static size_t configured[64] = {0};
    static size_t occ_smem[64][8] = {};
    static int occ_val[64][8] = {};
    const int dev = w.device;
    if (dev < 0 || dev >= 64) return set_error(Q35_ERR_INVALID, "gemv: device ordinal out of range");
    if (configured[dev] < smem) {
        int optin = 0;
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        if ((int)smem > optin) return set_error(Q35_ERR_INVALID, "gemv: K too large for the shared-memory activation image");
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
        if (e != cudaSuccess) return set_error(Q35_ERR_CUDA, std::string("gemv: shared memory ") + cudaGetErrorString(e));
        // clusters of up to 16 CTAs for the split per-group form
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return set_error(Q35_ERR_CUDA, std::string("gemv: cluster size ") + cudaGetErrorString(e));
        // every variant asks for the same (largest) shared-memory carveout, so consecutive
        // launches of different variants need no reconfiguration of the SMs between them
        e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        if (e != cudaSuccess) return set_error(Q35_ERR_CUDA, std::string("gemv: carveout ") + cudaGetErrorString(e));
        configured[dev] = (size_t)optin;
    }
    per_sm = 0;
    for (int i = 0; i < 8; ++i)
        if (occ_smem[dev][i] == smem) { per_sm = occ_val[dev][i]; return Q35_OK; }
    Q35_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, GEMV_THREADS, smem));
    for (int i = 7; i > 0; --i) { occ_smem[dev][i] = occ_smem[dev][i - 1]; occ_val[dev][i] = occ_val[dev][i - 1]; }
    occ_smem[dev][0] = smem;
    occ_val[dev][0] = per_sm;
    if (per_sm < 1) return set_error(Q35_ERR_INVALID, "gemv: K too large for the shared-memory activation image");
    return Q35_OK;
}

template <int FMT, int MT, int D>
static int launch_d(const GemvParams &p, size_t smem, int64_t grid, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)std::max<int64_t>(grid, 1));
    cfg.blockDim = dim3(GEMV_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (p.per_group && p.split > 1) {
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = (unsigned)p.split;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        cfg.numAttrs = 2;
    }
    Q35_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemv_kernel<FMT, MT, D>, p));
    return Q35_OK;
}

// Launch shape.  When every column group fits on the GPU at once (2-stage rings), one CTA
// per column group with the K range split over its warps and reduced in shared memory:
// no split-K workspace round trip, which is most of a small matmul's time.  When that
// leaves most SMs idle (few column groups: k/v, tensor-parallel shards), each column
// group's k-blocks are shared by the S CTAs of a thread-block cluster (S the largest
// power of two up to 16, at most the k-block count, with CG * S at most the SM count;
// one row chunk only), each staging only its share of the activation image, and the S
// partial sums meet in CTA 0's shared memory (exact).  Otherwise the balanced stream over all resident CTAs, with
// 3-stage rings where two CTAs still fit on an SM and 2-stage rings where they would not
// (large K: the activation image grows).
template <int FMT, int MT>
static int launch_t(const Weights &w, const GemvParams &p, cudaStream_t s) {
    const int sms = sm_count(w.device);
    size_t smem2 = 0, smem3 = 0;
    int ps2 = 0, ps3 = 0;
    int st = occupancy<FMT, MT, 2>(w, smem2, ps2);
    if (st) return st;
    GemvParams q = p;
    q.split = 1;
    if ((int64_t)w.CG <= (int64_t)ps2 * sms) {
        q.per_group = 1;
        const bool one_chunk = ceil_div(p.M, MT) == 1;
        for (int S = 16; S >= 2 && one_chunk; S /= 2) {
            // at most one CTA per SM: two split CTAs on one SM measured slower than one
            if (S > w.KB || (int64_t)w.CG * S > (int64_t)sms) continue;
            size_t smemS = 0;
            int psS = 0;
            if (occupancy<FMT, MT, 2>(w, smemS, psS, (int)ceil_div(w.KB, S), S) != Q35_OK) continue;
            if ((int64_t)w.CG * S > (int64_t)psS * sms) continue;
            q.split = S;
            return launch_d<FMT, MT, 2>(q, smemS, (int64_t)w.CG * S, s);
        }
        return launch_d<FMT, MT, 2>(q, smem2, w.CG, s);
    }
    q.per_group = 0;
    const int64_t units = (int64_t)w.CG * w.KB;
    st = occupancy<FMT, MT, 3>(w, smem3, ps3);
    if (!st && ps3 >= 2)
        return launch_d<FMT, MT, 3>(q, smem3, std::min<int64_t>((int64_t)ps3 * sms, ceil_div(units, GEMV_WARPS)), s);
    return launch_d<FMT, MT, 2>(q, smem2, std::min<int64_t>((int64_t)ps2 * sms, ceil_div(units, GEMV_WARPS)), s);
}

int launch_gemv(const Weights &w, const GemvArgs &a, Workspace &ws, cudaStream_t s) {
    if (a.M <= 0 || a.M > 64) return set_error(Q35_ERR_INVALID, "gemv: M must be in [1,64]");
    if (w.K > GEMV_MAX_K) return set_error(Q35_ERR_INVALID, "gemv: K above 131072");
    GemvParams p;
    p.tiles = reinterpret_cast<const uint4 *>(w.tiles);
    p.scales = w.scales;
    p.offsets = w.offsets;
    p.KB = w.KB; p.CG = w.CG; p.N = w.N; p.K = w.K;
    p.x = a.x; p.sx_row = a.sx_row; p.sx_k = a.sx_k; p.M = a.M;
    p.C = a.C; p.y = a.y; p.so_row = a.so_row; p.so_col = a.so_col;
    p.res = a.res;
    p.ws_acc = ws.acc;
    p.counters = ws.tickets;
    p.err = ws.err;
    p.per_group = 0;
    p.split = 1;
    p.sq = a.swiglu_q;
    if (p.sq && (w.N % 2)) return set_error(Q35_ERR_INVALID, "gemv: SwiGLU output needs interleaved column pairs");
    p.has_rope = a.rope ? 1 : 0;
    if (a.rope) {
        const GemvRope &g = *a.rope;
        if (p.sq || g.D <= 0 || (g.D % 2) || (int64_t)(g.H + 2 * g.KVH) * g.D != w.N || !g.q || !g.kc || !g.vc ||
            !g.row_seq || !g.row_i || !g.cache_pos || !g.cs)
            return set_error(Q35_ERR_INVALID, "gemv: q|k|v epilogue needs N = (H + 2 KVH) D, D even, every buffer");
        p.rope = g;
    }
    p.vec_x = (a.sx_k == 1 && (reinterpret_cast<uintptr_t>(a.x) & 7) == 0 &&
               (a.M == 1 || (a.sx_row % 8) == 0)) ? 1 : 0;
    p.bulk_x = (a.sx_k == 1 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 && (w.K % 16) == 0 &&
                (a.M == 1 || (a.sx_row % 16) == 0)) ? 1 : 0;
    if (!ws.acc || !ws.err || ws.acc_elems < gemv_workspace_acc_elems(w, a.M) || !ws.tickets ||
        ws.n_tickets < gemv_workspace_tickets(w))
        return set_error(Q35_ERR_STATE, "gemv: split-K workspace too small");
    const bool f35 = w.format == Q35_FMT_3P5BIT;
    switch (fit_mt(w, a.M)) {
        case 1: return f35 ? launch_t<Q35_FMT_3P5BIT, 1>(w, p, s) : launch_t<Q35_FMT_INT4, 1>(w, p, s);
        case 2: return f35 ? launch_t<Q35_FMT_3P5BIT, 2>(w, p, s) : launch_t<Q35_FMT_INT4, 2>(w, p, s);
        default: return f35 ? launch_t<Q35_FMT_3P5BIT, 4>(w, p, s) : launch_t<Q35_FMT_INT4, 4>(w, p, s);
    }
}

}  // namespace q35
