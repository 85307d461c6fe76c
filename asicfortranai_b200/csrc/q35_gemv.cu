// q35_gemv.cu -- decode GEMV / skinny GEMM on CUDA cores (dp4a), exact int32.
//
// Computes, for the reference kernels matmul_3p5bit_awq (matmul_3p5bit_dynamic.f90:42-64)
// and matmul_int4_awq (matmul_int4_groq.f90:117-137):
//   C(i,j) = sum_k A(i,k) * code(k,j)          (int32, exact)
//   y(i,j) = (float(C) + offset_j) * scale_j   (3.5-bit, :80)   or  float(C) * scale_j (INT4)
//
// Two launch shapes.  Per column group (when all column groups fit on the GPU at once):
// CTA b takes column group b, its warps split the k-blocks and add their exact partial
// sums in shared memory.  Stream (larger N): the grid holds as many CTAs as fit on the GPU
// at once; the (column group, k-block) tiles, stored column-group major, are cut into one
// contiguous range per warp of equal length, so every warp streams the same number of
// bytes and no wave tail is left.  A warp walks its range through a private ring of
// shared-memory stages; lane 0 fills each stage with one TMA bulk copy
// (cp.async.bulk, a whole 3.5 KB / 4 KB tile, completion counted on an mbarrier), so
// several tiles per warp are in flight without occupying registers or per-thread
// request slots.  Each lane owns one output column.  Launched with programmatic
// dependent launch: a CTA initialises its barriers and starts its weight stream before
// waiting (griddepcontrol.wait) for the kernel ahead of it, so the weight fetch of
// consecutive matmuls overlaps the previous kernel's tail.  Every mbarrier wait is bounded:
// when it gives up the kernel records Q35_ERR_TIMEOUT in the workspace error word,
// drains its own copies (again bounded) and leaves.
//
// The CTA first stages its activation rows for the whole K in shared memory in the
// even/odd image order and the per-k-block bias corrections (codes are stored biased,
// so sum a*code = sum a*biased - sum a*bias, see q35_internal.cuh).
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
    int per_group;           // one CTA per column group, K split over its warps (no workspace)
    int8_t *sq;              // SwiGLU output [M][N/2] int8 (interleaved gate/up columns), or null
    int *err;                // device error word (Q35_ERR_TIMEOUT on a failed wait)
    const float *res;        // optional residual: y = res + dequant(C), same strides as y
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

__device__ __forceinline__ float dequant(int FMT, int32_t c, const float *scales,
                                         const float *offsets, int64_t j) {
    float f = __int2float_rn(c);
    if (FMT == Q35_FMT_3P5BIT) return __fmul_rn(__fadd_rn(f, offsets[j]), scales[j]);
    return __fmul_rn(f, scales[j]);
}

// epilogue store of one output: C, and y = dequant (+ residual, the layer's x + f(x),
// transformer_layer.f90:550 and :557)
template <int FMT>
__device__ __forceinline__ void store_out(const GemvParams &p, int row, int64_t j, int32_t c) {
    const int64_t o = row * p.so_row + j * p.so_col;
    if (p.C) p.C[o] = c;
    if (p.y) {
        float v = dequant(FMT, c, p.scales, p.offsets, j);
        if (p.res) v = __fadd_rn(p.res[o], v);
        p.y[o] = v;
    }
}

// one row's outputs of a warp's 32 columns (j = this lane's column, valid = j < N); every
// lane of the warp calls it.  With sq set the columns are (gate, up) pairs: the even lane
// forms silu(gate) * up (swiglu_kernel, transformer_layer.f90:212-229) and its int8 value.
template <int FMT>
__device__ __forceinline__ void store_row(const GemvParams &p, int row, int64_t j, int32_t c, bool valid) {
    if (p.sq) {
        const float v = valid ? dequant(FMT, c, p.scales, p.offsets, j) : 0.0f;
        const float up = __shfl_xor_sync(0xffffffffu, v, 1);
        if (valid && (j & 1) == 0) {
            const float sw = __fdiv_rn(v, __fadd_rn(1.0f, q35_expf(-v)));
            p.sq[(int64_t)row * (p.N / 2) + (j >> 1)] = quant127(__fmul_rn(sw, up));
        }
    } else if (valid) {
        store_out<FMT>(p, row, j, c);
    }
}

template <int FMT>
struct Tile {
    static constexpr int NC = (FMT == Q35_FMT_3P5BIT) ? 7 : 8;    // 16-byte chunks per lane
    static constexpr int BYTES = NC * 512;
    static constexpr int U4 = NC * 32;
};

template <int FMT, int MT, int D>
__global__ void __launch_bounds__(GEMV_THREADS, 1)
gemv_kernel(const GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    using T = Tile<FMT>;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int KB = p.KB;
    // layout: [ring: warps x D tiles][img: MT x KB x 256 B][corr: MT x KB int][mbarriers]
    //         [red: warps x MT x 32 int, one-CTA-per-column-group mode]
    uint8_t *ring = smem + (size_t)warp * D * T::BYTES;
    uint32_t *img = reinterpret_cast<uint32_t *>(smem + (size_t)GEMV_WARPS * D * T::BYTES);
    int32_t *corr = reinterpret_cast<int32_t *>(reinterpret_cast<uint8_t *>(img) + (size_t)MT * KB * KBLK);
    const uint32_t bars = (uint32_t)__cvta_generic_to_shared(
        reinterpret_cast<uint8_t *>(corr) + round_up((int64_t)MT * KB * 4, 8)) + warp * D * 8;
    int32_t *red = reinterpret_cast<int32_t *>(reinterpret_cast<uint8_t *>(corr) + round_up((int64_t)MT * KB * 4, 8) +
                                               GEMV_WARPS * D * 8);
    const uint32_t ring_s = (uint32_t)__cvta_generic_to_shared(ring);
    const uint8_t *gtiles = reinterpret_cast<const uint8_t *>(p.tiles);

    const int64_t U = (int64_t)p.CG * KB;
    const int64_t Wt = (int64_t)gridDim.x * GEMV_WARPS;
    const int64_t gw = (int64_t)blockIdx.x * GEMV_WARPS + warp;
    // stream mode: one balanced range of tiles per warp across the grid; per-group mode:
    // CTA b takes column group b and its warps split the k-blocks
    const int64_t u0 = p.per_group ? (int64_t)blockIdx.x * KB + (int64_t)KB * warp / GEMV_WARPS : U * gw / Wt;
    const int64_t u1 = p.per_group ? (int64_t)blockIdx.x * KB + (int64_t)KB * (warp + 1) / GEMV_WARPS : U * (gw + 1) / Wt;
    const int64_t Np = (int64_t)p.CG * 32;
    const int nchunks = (p.M + MT - 1) / MT;

    if (lane == 0) {
        for (int s = 0; s < D; ++s) mbar_init(bars + 8 * s, 1);
        mbar_fence_init();
    }
    __syncwarp();
    // programmatic dependent launch: let the next kernel in the stream begin its own
    // weight stream as our CTAs retire
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    uint32_t phase = 0;       // bit s: parity of the next completion of stage s
    bool failed = false;

    for (int chunk = 0; chunk < nchunks; ++chunk) {
        const int r0 = chunk * MT;
        // ---- first tiles of this warp's range: in flight while activations are staged ----
        if (lane == 0 && !failed) {
            for (int s = 0; s < D && u0 + s < u1; ++s) {
                mbar_expect_tx(bars + 8 * s, T::BYTES);
                bulk_g2s(ring_s + s * T::BYTES, gtiles + (size_t)(u0 + s) * T::BYTES, T::BYTES, bars + 8 * s);
            }
            for (int s = D; s < D + Q35_GEMV_PF && u0 + s < u1; ++s)
                bulk_prefetch_l2(gtiles + (size_t)(u0 + s) * T::BYTES, T::BYTES);
        }
        // weights never depend on the previous kernel; activations, the workspace and the
        // outputs may: wait for the predecessor grid here (a no-op without one)
        if (chunk == 0) asm volatile("griddepcontrol.wait;" ::: "memory");
        // ---- stage the activation image of rows r0.., all k-blocks, and corrections ----
        // (loads of up to 8 items per warp are issued before any is used)
        for (int t0 = warp; t0 < MT * KB; t0 += 8 * GEMV_WARPS) {
            uint32_t lo[8], hi[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int t = t0 + i * GEMV_WARPS;
                lo[i] = 0;
                hi[i] = 0;
                if (t >= MT * KB) continue;
                const int r = t / KB, kb = t % KB, row = r0 + r;
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
                if (t >= MT * KB) break;
                const int r = t / KB, kb = t % KB;
                const uint32_t e = __byte_perm(lo[i], hi[i], 0x6420);   // k0, k0+2, k0+4, k0+6
                const uint32_t o = __byte_perm(lo[i], hi[i], 0x7531);   // k0+1, k0+3, k0+5, k0+7
                uint32_t *im = img + ((size_t)r * KB + kb) * 64;
                im[lane] = e;
                im[32 + lane] = o;
                int c = (FMT == Q35_FMT_3P5BIT) ? __dp4a((int)e, 0x08080808, __dp4a((int)o, 0x04040404, 0))
                                                : __dp4a((int)e, 0x08080808, __dp4a((int)o, 0x08080808, 0));
#pragma unroll
                for (int s = 16; s > 0; s >>= 1) c += __shfl_xor_sync(0xffffffffu, c, s);
                if (lane == 0) corr[r * KB + kb] = c;
            }
        }
        __syncthreads();

        if (u0 < u1 && !failed) {
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
                    const uint32_t *im = img + ((size_t)r * KB + kb) * 64;
                    if (FMT == Q35_FMT_3P5BIT) dot35(W, im, acc[r]); else dot4(W, im, acc[r]);
                    csum[r] += corr[r * KB + kb];
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
                            if (row < p.M) store_row<FMT>(p, row, j, tot[r], j < p.N);
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
                            store_row<FMT>(p, row, j, j < p.N ? atomicExch(&p.ws_acc[row * Np + j], 0) : 0, j < p.N);
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
            for (int r = warp; r < MT; r += GEMV_WARPS) {
                int t = 0;
#pragma unroll
                for (int w2 = 0; w2 < GEMV_WARPS; ++w2) t += red[(w2 * MT + r) * 32 + lane];
                const int64_t j = (int64_t)blockIdx.x * 32 + lane;
                const int row = r0 + r;
                if (row < p.M) store_row<FMT>(p, row, j, t, j < p.N);
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

static size_t smem_bytes(int fmt, int MT, int D, int KB);

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

static size_t smem_bytes(int fmt, int MT, int D, int KB) {
    const size_t tb = fmt == Q35_FMT_3P5BIT ? Tile<Q35_FMT_3P5BIT>::BYTES : Tile<Q35_FMT_INT4>::BYTES;
    return (size_t)GEMV_WARPS * D * tb + (size_t)MT * KB * KBLK + round_up((int64_t)MT * KB * 4, 8) +
           (size_t)GEMV_WARPS * D * 8 + (size_t)GEMV_WARPS * MT * 32 * 4;
}

size_t gemv_workspace_acc_elems(const Weights &w, int32_t M) { return (size_t)M * w.CG * 32; }

size_t gemv_workspace_tickets(const Weights &w) {
    return (size_t)w.CG * ((64 + GEMV_MT_MAX - 1) / GEMV_MT_MAX);
}

// shared-memory size and CTAs per SM of gemv_kernel<FMT, MT, D> for K-blocks KB (the
// dynamic shared-memory limit raised once per device, occupancies cached)
template <int FMT, int MT, int D>
static int occupancy(const Weights &w, size_t &smem, int &per_sm) {
    auto kern = gemv_kernel<FMT, MT, D>;
    smem = smem_bytes(FMT, MT, D, w.KB);
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
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    Q35_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemv_kernel<FMT, MT, D>, p));
    return Q35_OK;
}

// Launch shape.  When every column group fits on the GPU at once (2-stage rings), one CTA
// per column group with the K range split over its warps and reduced in shared memory:
// no split-K workspace round trip, which is most of a small matmul's time.  Otherwise the
// balanced stream over all resident CTAs, with 3-stage rings where two CTAs still fit on
// an SM and 2-stage rings where they would not (large K: the activation image grows).
template <int FMT, int MT>
static int launch_t(const Weights &w, const GemvParams &p, cudaStream_t s) {
    const int sms = sm_count(w.device);
    size_t smem2 = 0, smem3 = 0;
    int ps2 = 0, ps3 = 0;
    int st = occupancy<FMT, MT, 2>(w, smem2, ps2);
    if (st) return st;
    GemvParams q = p;
    if ((int64_t)w.CG <= (int64_t)ps2 * sms) {
        q.per_group = 1;
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
    p.sq = a.swiglu_q;
    if (p.sq && (w.N % 2)) return set_error(Q35_ERR_INVALID, "gemv: SwiGLU output needs interleaved column pairs");
    p.vec_x = (a.sx_k == 1 && (reinterpret_cast<uintptr_t>(a.x) & 7) == 0 &&
               (a.M == 1 || (a.sx_row % 8) == 0)) ? 1 : 0;
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
