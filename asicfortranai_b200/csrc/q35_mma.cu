// q35_mma.cu -- skinny and prefill GEMM on the 5th-generation tensor cores
// (tcgen05.mma kind::i8, int32 accumulators in tensor memory), exact int32.
//
// Same contract as the CUDA-core GEMV (q35_gemv.cu): for the reference kernels
// matmul_3p5bit_awq (matmul_3p5bit_dynamic.f90:42-64) and matmul_int4_awq
// (matmul_int4_groq.f90:117-137)
//   C(i,j) = sum_k A(i,k) * code(k,j)          (int32, exact)
//   y(i,j) = (float(C) + offset_j) * scale_j   (3.5-bit)   or  float(C) * scale_j (INT4)
// for M >= 5 activation rows (decode batches, the skinny sweep, prefill).
//
// Tile: 128 weight columns (the MMA's M, four column groups of the resident tile format)
// x BN activation rows (the MMA's N, a multiple of 16 up to 256).  Per 256-k block:
//   * weight producer (warp 0): four cp.async.bulk copies of the packed column-group
//     tiles into a ring of packed stages (issued before waiting on the previous kernel:
//     the weights do not depend on it);
//   * activation producer (warp 2): two 2D TMA loads (128 k x BN rows each, 128-byte
//     swizzle, rows past M and k past K read as zero) into the B operand of the stage;
//   * converters (warps 8-23, two sets of 8 taking alternate k-blocks, so that two
//     k-blocks are converted at once): decode the biased codes into unsigned bytes in k order
//     and write them with tcgen05.st straight into a tensor-memory A stage (row = weight
//     column = lane, four k values per 32-bit column; warp 8+c: column group c&3 -- the
//     lane quarter the warp may access -- k half (c>>2)&1, k-block parity c>>3); 3.5-bit
//     costs ~0.85 integer
//     ops per weight, INT4 ~0.6.  Keeping the decoded operand out of shared memory
//     spares the generic-to-async proxy fence a shared-memory operand would need per
//     stage, which cost about a microsecond per k-block;
//   * MMA issuer (warp 1, one thread): 8 x tcgen05.mma (K=32 each, unsigned A from
//     tensor memory x signed B from shared memory), then tcgen05.commit frees the stage.
//     The issue alone takes ~0.5 us per k-block, the pipeline's slowest step at BN <= 64,
//     so there a second issuer (warp 3) takes every other k-block into an accumulator of
//     its own and the epilogue adds the two;
//   * epilogue (warps 4-7, one per 32-lane quarter of tensor memory): tcgen05.ld of the
//     accumulator, minus the row's bias correction sum_k a_k*bias_k (computed by
//     rowcorr_kernel ahead of the GEMM), dequant, store.
// Tensor memory holds two accumulator buffers (so the epilogue of one tile overlaps the
// main loop of the next), each of one or two (two issuers) accumulators, and the A stages:
// 2*BN (or 4*BN) + 64*S <= 512 columns.
//
// Work split: the (tile, k-block) list, tiles ordered column-tile major so that the row
// tiles of one weight tile run side by side and share it through L2, is cut into one
// contiguous range per CTA (one CTA per SM).  A tile cut by a range boundary is
// finished through a split slot: its pieces add their exact partial sums into the slot
// of the CTA owning its first k-block (red.add: integer addition is order free), count
// their k-blocks on the slot's ticket (release/acquire), and the piece completing the
// count reads the totals back with atomicExch(.., 0) -- leaving the slot zero -- and runs
// the epilogue.
//
// Every wait is bounded: a wait that gives up records Q35_ERR_TIMEOUT in the workspace
// error word and raises a shared abort flag that ends the other roles' waits; before the
// CTA leaves, the producers wait (bounded) for their copies in flight, the MMA thread
// for its MMAs, and tensor memory is released.  Launched with programmatic dependent
// launch; everything that reads activations or the row corrections, or writes any output,
// runs after griddepcontrol.wait.
#include <cuda.h>

#include <algorithm>

#include "q35_internal.cuh"

namespace q35 {

constexpr int MMA_THREADS = 768;         // 24 warps
constexpr int MMA_BM = 128;                 // weight columns per tile
constexpr int A_COLS = KBLK / 4;            // tensor-memory columns of one decoded k-block
constexpr int MMA_BN_MAX = 128;             // rows per tile (tensor memory: 2*BN + 64*S <= 512)
constexpr uint32_t WAIT_LIMIT = 1u << 26;

struct MmaParams {
    const uint8_t *tiles;
    const float *scales, *offsets;
    int32_t KB, CG, N, K, M;
    int32_t BN, RT, CT;        // rows per tile, row tiles, column tiles
    int64_t per, work;         // k-blocks per CTA, total k-blocks
    int32_t S, SB, P;          // decoded-weight (tensor memory) stages, activation stages, packed stages
    uint32_t tile_bytes;
    uint32_t tmem_cols;
    int32_t *C;
    float *y;
    const float *res;
    int64_t so_row, so_col;
    const int32_t *corr;       // [M]
    int32_t *ws;               // [grid][BN][128], zero between calls
    uint32_t *tickets;         // [grid][4], zero between calls
    int *err;
    uint32_t off_b, off_pk, off_bar;   // byte offsets inside the aligned dynamic smem
    uint32_t a_col0;                    // first tensor-memory column of the A stages
    int32_t dual;                       // two MMA issuers (warps 1 and 3) taking alternate
                                        // k-blocks into their own accumulators
};

// ---- PTX wrappers ------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
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
// bounded wait; gives up when the limit passes or another role raised the abort flag
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int *abort_flag) {
    for (uint32_t i = 0; i < WAIT_LIMIT; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 255u && *abort_flag) return false;
    }
    return false;
}
// bounded wait for roles that wait long and are off the critical loop (epilogue, the
// accumulator hand-back, the producers' slot waits): sleeps between polls so that the
// spinning warps do not take issue slots from the converters
__device__ __forceinline__ bool mbar_wait_lazy(uint32_t bar, uint32_t parity, volatile int *abort_flag) {
    for (uint32_t i = 0; i < (1u << 22); ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        __nanosleep(i < 16 ? 32 : 256);
    }
    return false;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int32_t x, int32_t y,
                                            uint32_t bar) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%2, %3}], [%4];"
                 ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(bar) : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]; unsigned 8-bit A, signed 8-bit B, s32 D
__device__ __forceinline__ void tc_mma_i8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}"
                 ::"r"(d_tmem), "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}
// 32 consecutive columns of this thread's lane, then wait for the stores to complete
__device__ __forceinline__ void tc_st32(uint32_t taddr, const uint4 (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0],"
                 " {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16,"
                 " %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
                 ::"r"(taddr), "r"(v[0].x), "r"(v[0].y), "r"(v[0].z), "r"(v[0].w), "r"(v[1].x), "r"(v[1].y),
                   "r"(v[1].z), "r"(v[1].w), "r"(v[2].x), "r"(v[2].y), "r"(v[2].z), "r"(v[2].w), "r"(v[3].x),
                   "r"(v[3].y), "r"(v[3].z), "r"(v[3].w), "r"(v[4].x), "r"(v[4].y), "r"(v[4].z), "r"(v[4].w),
                   "r"(v[5].x), "r"(v[5].y), "r"(v[5].z), "r"(v[5].w), "r"(v[6].x), "r"(v[6].y), "r"(v[6].z),
                   "r"(v[6].w), "r"(v[7].x), "r"(v[7].y), "r"(v[7].z), "r"(v[7].w)
                 : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tc_ld16(uint32_t taddr, int32_t (&v)[16]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32"
                 " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                   "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
                   "=r"(v[14]), "=r"(v[15])
                 : "r"(taddr) : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned *p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ void red_add(int32_t *p, int32_t v) {
    asm volatile("red.relaxed.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// K-major operand with 128-byte swizzle: rows of 128 bytes (128 k values), 8-row atoms
// of 1024 bytes (the stride byte offset); the leading byte offset is unused in this mode
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
    return (uint64_t)((addr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// instruction descriptor: D s32, A unsigned 8-bit, B signed 8-bit, both K-major, M=128
__host__ __device__ constexpr uint32_t idesc_i8(int BN) {
    return (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(MMA_BM >> 4) << 24);
}

// position in a ring of mbarrier-guarded stages: index and the phase parity of its
// current use
struct Ring {
    int i = 0;
    uint32_t ph = 0;
    __device__ __forceinline__ void next(int n) {
        if (++i == n) { i = 0; ph ^= 1u; }
    }
    // the entry used j steps ago (1 <= j <= n)
    __device__ __forceinline__ Ring back(int j, int n) const {
        Ring r;
        r.i = i - j;
        r.ph = ph;
        if (r.i < 0) { r.i += n; r.ph ^= 1u; }
        return r;
    }
};

__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t s) { return __byte_perm(a, b, s); }

// 3.5-bit: one group of 32 pairs (words W[O..O+6]) -> 64 codes in k order, 4 chunks.
// Byte b of word i holds pair 4i+b's field b2 | b1<<3 and bit i of pair 28+b's field.
template <int O>
__device__ __forceinline__ void dec35_group(const uint32_t (&W)[16], uint4 (&out)[4]) {
    uint32_t hi[8], lo[8], F = 0;
#pragma unroll
    for (int i = 0; i < 7; ++i) {
        const uint32_t w = W[O + i];
        F |= ((w >> 7) & 0x01010101u) << i;
        lo[i] = w & 0x07070707u;            // odd-k codes b2 of pairs 4i..4i+3
        hi[i] = (w >> 3) & 0x0F0F0F0Fu;     // even-k codes b1
    }
    lo[7] = F & 0x07070707u;
    hi[7] = (F >> 3) & 0x0F0F0F0Fu;
#pragma unroll
    for (int j = 0; j < 4; ++j)
        out[j] = make_uint4(prmt(hi[2 * j], lo[2 * j], 0x5140), prmt(hi[2 * j], lo[2 * j], 0x7362),
                            prmt(hi[2 * j + 1], lo[2 * j + 1], 0x5140), prmt(hi[2 * j + 1], lo[2 * j + 1], 0x7362));
}

// INT4: plane words E (even k) / O (odd k) of pairs 8w..8w+7 -> 16 codes in k order
__device__ __forceinline__ uint4 dec4_chunk(uint32_t E, uint32_t O) {
    const uint32_t el = E & 0x0F0F0F0Fu, eh = (E >> 4) & 0x0F0F0F0Fu;
    const uint32_t ol = O & 0x0F0F0F0Fu, oh = (O >> 4) & 0x0F0F0F0Fu;
    return make_uint4(prmt(el, ol, 0x5140), prmt(el, ol, 0x7362), prmt(eh, oh, 0x5140), prmt(eh, oh, 0x7362));
}

template <int FMT>
__device__ __forceinline__ void store_one(const MmaParams &p, int row, int col, int32_t c) {
    const int64_t o = row * p.so_row + (int64_t)col * p.so_col;
    if (p.C) p.C[o] = c;
    if (p.y) {
        const float f = __int2float_rn(c);
        float v = (FMT == Q35_FMT_3P5BIT) ? __fmul_rn(__fadd_rn(f, p.offsets[col]), p.scales[col])
                                          : __fmul_rn(f, p.scales[col]);
        if (p.res) v = __fadd_rn(p.res[o], v);
        p.y[o] = v;
    }
}

// DUAL: two MMA issuers (p.dual), a compile-time choice so that the one-issuer form
// (prefill tiles) carries none of the second issuer's branches
template <int FMT, bool DUAL>
__global__ void __launch_bounds__(MMA_THREADS, 1)
mma_kernel(const MmaParams p, const __grid_constant__ CUtensorMap xmap) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t *sbase = smem_raw + (base - raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int S = p.S, P = p.P, BN = p.BN;

    // barriers: pk_full[P] pk_empty[P] a_full[S] op_empty[S] b_full[SB] b_empty[SB] acc_full[2]
    // acc_empty[2] drain.  The activation ring is deeper than the tensor-memory A ring: its
    // loads are issued many k-blocks ahead, so their latency under the weight stream's load
    // stays off the MMA's path.  A tcgen05.commit tracks all prior MMAs of the thread, so
    // one commit per ring frees both stages of a k-block.
    const int SB = p.SB;
    const uint32_t bars = base + p.off_bar;
    auto pk_full = [&](int i) { return bars + 8u * i; };
    auto pk_empty = [&](int i) { return bars + 8u * (P + i); };
    auto a_full = [&](int i) { return bars + 8u * (2 * P + i); };
    auto op_empty = [&](int i) { return bars + 8u * (2 * P + S + i); };
    auto b_full = [&](int i) { return bars + 8u * (2 * P + 2 * S + i); };
    auto b_empty = [&](int i) { return bars + 8u * (2 * P + 2 * S + SB + i); };
    const int nb0 = 2 * P + 2 * S + 2 * SB;
    auto acc_full = [&](int i) { return bars + 8u * (nb0 + i); };
    auto acc_empty = [&](int i) { return bars + 8u * (nb0 + 2 + i); };
    const uint32_t drain_bar = bars + 8u * (nb0 + 4);
    uint8_t *misc = sbase + p.off_bar + 8 * (nb0 + 5);
    volatile uint32_t *tmem_slot = reinterpret_cast<volatile uint32_t *>(misc);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(misc + 4);

    if (tid == 0) {
        for (int i = 0; i < P; ++i) { mbar_init(pk_full(i), 1); mbar_init(pk_empty(i), 8); }
        for (int i = 0; i < S; ++i) { mbar_init(a_full(i), 8); mbar_init(op_empty(i), 1); }
        for (int i = 0; i < SB; ++i) { mbar_init(b_full(i), 1); mbar_init(b_empty(i), 1); }
        for (int i = 0; i < 2; ++i) { mbar_init(acc_full(i), DUAL ? 2 : 1); mbar_init(acc_empty(i), 4); }
        mbar_init(drain_bar, DUAL ? 2 : 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {   // tensor memory for two accumulator buffers of BN columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32((const void *)tmem_slot)), "r"(p.tmem_cols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 64) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&xmap)) : "memory");
    pdl_trigger();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int64_t beg = (int64_t)blockIdx.x * p.per;
    const int64_t end = min64(p.work, beg + p.per);
    const int KB = p.KB;
    bool ok = true;
    auto fail = [&]() {
        ok = false;
        *abort_flag = 1;
        atomicExch(p.err, Q35_ERR_TIMEOUT);
    };

    // Every role walks the same segment list -- (tile, k-block range) pieces of the CTA's
    // range -- with one division at the start; ring positions and phases advance by
    // increments (a 64-bit division per k-block costs as much as the k-block's MMAs).
    const int64_t t_beg = beg / KB;
    const int kb_beg = (int)(beg - t_beg * KB);
    const int ct_beg = (int)(t_beg / p.RT), rt_beg = (int)(t_beg - (int64_t)ct_beg * p.RT);

    if (warp == 0) {
        // ---------------- weight producer ----------------
        // lane 0 waits for a free slot and arms its barrier; lanes 0..3 then issue one
        // column group's bulk copy each (one thread issuing every copy could not keep
        // enough bytes in flight)
        if (lane < 4) {
            Ring pk{};
            int64_t issued = 0;
            int ct = ct_beg, rt = rt_beg, kb0 = kb_beg;
            for (int64_t u = beg; u < end && ok;) {
                const int n = (int)min64(KB - kb0, end - u);
                const int ng = min(4, p.CG - 4 * ct);
                for (int kb = kb0; kb < kb0 + n && ok; ++kb) {
                    bool got = true;
                    if (lane == 0) {
                        got = mbar_wait_lazy(pk_empty(pk.i), pk.ph ^ 1u, abort_flag);
                        if (got) mbar_expect_tx(pk_full(pk.i), (uint32_t)ng * p.tile_bytes);
                    }
                    if (!__shfl_sync(0xfu, (int)got, 0)) { fail(); break; }
                    if (lane < ng)
                        bulk_g2s(base + p.off_pk + (uint32_t)pk.i * 4u * p.tile_bytes + (uint32_t)lane * p.tile_bytes,
                                 p.tiles + ((size_t)(4 * ct + lane) * KB + kb) * p.tile_bytes, p.tile_bytes,
                                 pk_full(pk.i));
                    pk.next(P);
                    ++issued;
                }
                u += n;
                kb0 = 0;
                if (++rt == p.RT) { rt = 0; ++ct; }
            }
            // copies in flight land before the CTA leaves
            if (lane == 0)
                for (int j = 1; j <= min64(P, issued); ++j) {
                    const Ring e = pk.back(j, P);
                    if (!mbar_wait(pk_full(e.i), e.ph, abort_flag)) { fail(); break; }
                }
        }
    } else if (warp == 2) {
        // ---------------- activation producer ----------------
        if (lane == 0) {
            pdl_wait();
            Ring st{};
            int64_t issued = 0;
            int rt = rt_beg, kb0 = kb_beg;
            for (int64_t u = beg; u < end && ok;) {
                const int n = (int)min64(KB - kb0, end - u);
                for (int kb = kb0; kb < kb0 + n && ok; ++kb) {
                    if (!mbar_wait_lazy(b_empty(st.i), st.ph ^ 1u, abort_flag)) { fail(); break; }
                    mbar_expect_tx(b_full(st.i), (uint32_t)BN * 256u);
                    const uint32_t dst = base + p.off_b + (uint32_t)st.i * (uint32_t)BN * 256u;
                    tma_load_2d(dst, &xmap, kb * KBLK, rt * BN, b_full(st.i));
                    tma_load_2d(dst + (uint32_t)BN * 128u, &xmap, kb * KBLK + 128, rt * BN, b_full(st.i));
                    st.next(SB);
                    ++issued;
                }
                u += n;
                kb0 = 0;
                if (++rt == p.RT) rt = 0;
            }
            for (int j = 1; j <= min64(SB, issued); ++j) {
                const Ring e = st.back(j, SB);
                if (!mbar_wait(b_full(e.i), e.ph, abort_flag)) { fail(); break; }
            }
        }
    } else if (warp == 1 || (warp == 3 && DUAL)) {
        // ---------------- MMA issuer(s) ----------------
        // one thread issues a k-block's 8 MMAs and ~0.5 us of its time goes into that issue
        // alone, so with dual set two threads (warps 1 and 3) take alternate k-blocks of the
        // CTA's range, each into its own accumulator of the tile's buffer (the epilogue adds
        // the two, integer addition being exact); without dual one thread takes them all
        if (lane == 0) {
            const int par = warp == 3 ? 1 : 0;
            const uint32_t idesc = idesc_i8(BN);
            Ring st{}, sb{};
            int kb0 = kb_beg;
            int64_t seg = 0, kix = 0;
            for (int64_t u = beg; u < end && ok; ++seg) {
                const int n = (int)min64(KB - kb0, end - u);
                const int buf = (int)(seg & 1);
                if (!mbar_wait_lazy(acc_empty(buf), (uint32_t)((seg >> 1) & 1) ^ 1u, abort_flag)) { fail(); break; }
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)((DUAL ? 2 * buf + par : buf) * BN);
                bool first = true;
                for (int i = 0; i < n && ok; ++i, ++kix) {
                    if (DUAL && (int)(kix & 1) != par) {   // the other issuer's k-block
                        st.next(S);
                        sb.next(SB);
                        continue;
                    }
                    if (!mbar_wait(a_full(st.i), st.ph, abort_flag) || !mbar_wait(b_full(sb.i), sb.ph, abort_flag)) {
                        fail();
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = tmem + p.a_col0 + (uint32_t)(st.i * A_COLS);
                    const uint32_t b0 = base + p.off_b + (uint32_t)sb.i * (uint32_t)BN * 256u;
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const uint32_t ko = (uint32_t)(j & 3) * 32u;
                        const uint64_t bd = smem_desc_sw128(b0 + (uint32_t)(j >> 2) * (uint32_t)BN * 128u + ko);
                        tc_mma_i8_ts(d, a0 + (uint32_t)(8 * j), bd, idesc, (!first || j > 0) ? 1u : 0u);
                    }
                    first = false;
                    tc_commit(op_empty(st.i));
                    tc_commit(b_empty(sb.i));
                    st.next(S);
                    sb.next(SB);
                }
                // (an issuer without a k-block in this piece arrives at once: its accumulator
                // is not read for the piece)
                if (ok) tc_commit(acc_full(buf));
                u += n;
                kb0 = 0;
            }
            // every MMA issued has completed before tensor memory is released
            tc_commit(drain_bar);
            if (!mbar_wait(drain_bar, 0, abort_flag)) fail();
        }
    } else if (warp >= 8) {
        // ---------------- converters ----------------
        const int cw = warp - 8, g = cw & 3, h = (cw >> 2) & 1, par = cw >> 3;
        Ring pk{}, st{};
        int64_t kix = 0;   // k-block index in the CTA's range: this set takes kix % 2 == par
        int ct = ct_beg, rt = rt_beg, kb0 = kb_beg;
        for (int64_t u = beg; u < end && ok;) {
            const int n = (int)min64(KB - kb0, end - u);
            const bool live = (4 * ct + g) < p.CG;
            for (int i = 0; i < n; ++i, ++kix) {
                if ((int)(kix & 1) != par) {   // the other set's k-block
                    pk.next(P);
                    st.next(S);
                    continue;
                }
                if (!__all_sync(0xffffffffu, mbar_wait(pk_full(pk.i), pk.ph, abort_flag))) {
                    fail();
                    break;
                }
                uint4 out[8];
                if (live) {
                    const uint8_t *src = sbase + p.off_pk + (size_t)pk.i * 4 * p.tile_bytes + (size_t)g * p.tile_bytes +
                                         (size_t)lane * 16;
                    uint32_t W[16];
                    if (FMT == Q35_FMT_3P5BIT) {
                        const int c0 = h ? 3 : 0;   // words 0..13 (groups 0,1) or 14..27 (groups 2,3)
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            const uint4 v = *reinterpret_cast<const uint4 *>(src + (size_t)(c0 + c) * 512);
                            W[4 * c] = v.x; W[4 * c + 1] = v.y; W[4 * c + 2] = v.z; W[4 * c + 3] = v.w;
                        }
                    } else {
                        // even plane chunks 2h, 2h+1 -> W[0..7]; odd plane chunks 4+2h, 5+2h -> W[8..15]
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            const int ch = (c < 2) ? 2 * h + c : 4 + 2 * h + (c - 2);
                            const uint4 v = *reinterpret_cast<const uint4 *>(src + (size_t)ch * 512);
                            W[4 * c] = v.x; W[4 * c + 1] = v.y; W[4 * c + 2] = v.z; W[4 * c + 3] = v.w;
                        }
                    }
                    if (FMT == Q35_FMT_3P5BIT) {
                        uint4 ga[4], gb[4];
                        if (h == 0) { dec35_group<0>(W, ga); dec35_group<7>(W, gb); }
                        else { dec35_group<2>(W, ga); dec35_group<9>(W, gb); }
#pragma unroll
                        for (int j = 0; j < 4; ++j) { out[j] = ga[j]; out[4 + j] = gb[j]; }
                    } else {
#pragma unroll
                        for (int j = 0; j < 8; ++j) out[j] = dec4_chunk(W[j], W[8 + j]);
                    }
                    // the decode above overlapped the MMAs still reading this stage
                    if (!__all_sync(0xffffffffu, mbar_wait(op_empty(st.i), st.ph ^ 1u, abort_flag))) {
                        fail();
                        break;
                    }
                    tc_fence_after();
                    // lane quarter g (this warp's), columns of stage st.i, k half h
                    tc_st32(tmem + ((uint32_t)(32 * g) << 16) + p.a_col0 + (uint32_t)(st.i * A_COLS + 32 * h), out);
                } else {
                    if (!__all_sync(0xffffffffu, mbar_wait(op_empty(st.i), st.ph ^ 1u, abort_flag))) {
                        fail();
                        break;
                    }
                }
                tc_fence_before();
                __syncwarp();
                // the packed stage is released only here, after the tensor-memory stores:
                // they use every word loaded from it, so no load of the stage is still in
                // flight when the next bulk copy may overwrite it
                if (lane == 0) {
                    mbar_arrive(pk_empty(pk.i));
                    mbar_arrive(a_full(st.i));
                }
                pk.next(P);
                st.next(S);
            }
            if (!ok) break;
            u += n;
            kb0 = 0;
            if (++rt == p.RT) { rt = 0; ++ct; }
        }
    } else if (warp >= 4) {
        // ---------------- epilogue ----------------
        // each warp owns one 32-lane quarter of tensor memory (32 weight columns) and
        // finishes its split pieces on its own ticket, so the four warps never wait on
        // one another
        const int q = warp & 3;
        const int colt = 32 * q + lane;    // column inside the tile = tensor-memory lane
        pdl_wait();
        int64_t seg = 0, t = t_beg, kix = 0;
        int ct = ct_beg, rt = rt_beg, kb0 = kb_beg;
        for (int64_t u = beg; u < end && ok; ++seg) {
            const int n = (int)min64(KB - kb0, end - u);
            const int buf = (int)(seg & 1);
            // with two issuers the piece's k-blocks alternate between two accumulators
            // (by their index in the CTA's range); a one-k-block piece fills only one
            const bool has0 = !DUAL || n >= 2 || (kix & 1) == 0;
            const bool has1 = DUAL && (n >= 2 || (kix & 1) == 1);
            kix += n;
            const int col = ct * MMA_BM + colt;
            const int row0 = rt * BN;
            const bool whole = (n == KB);
            const int64_t slot = (t * KB) / p.per;
            int32_t *wsl = p.ws + slot * (int64_t)BN * MMA_BM;
            if (!__all_sync(0xffffffffu, mbar_wait_lazy(acc_full(buf), (uint32_t)((seg >> 1) & 1), abort_flag))) {
                fail();
                break;
            }
            tc_fence_after();
            const uint32_t tbase = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)((DUAL ? 2 * buf : buf) * BN);
            for (int r0 = 0; r0 < BN; r0 += 16) {
                int32_t v[16];
                if (has0) {
                    tc_ld16(tbase + (uint32_t)r0, v);
                } else {
#pragma unroll
                    for (int i = 0; i < 16; ++i) v[i] = 0;
                }
                if (has1) {
                    int32_t v1[16];
                    tc_ld16(tbase + (uint32_t)(BN + r0), v1);
#pragma unroll
                    for (int i = 0; i < 16; ++i) v[i] += v1[i];
                }
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int row = row0 + r0 + i;
                    if (row < p.M && col < p.N) {
                        if (whole) store_one<FMT>(p, row, col, v[i] - p.corr[row]);
                        else red_add(wsl + (int64_t)(r0 + i) * MMA_BM + colt, v[i]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty(buf));
            if (!whole) {
                __threadfence();
                __syncwarp();
                unsigned last = 0;
                if (lane == 0) {
                    unsigned *tk = &p.tickets[slot * 4 + q];
                    last = (atom_add_acq_rel(tk, (unsigned)n) + (unsigned)n == (unsigned)KB) ? 1u : 0u;
                }
                last = __shfl_sync(0xffffffffu, last, 0);
                if (last) {
                    for (int rr = 0; rr < BN; ++rr) {
                        const int row = row0 + rr;
                        if (row >= p.M) break;
                        if (col < p.N)
                            store_one<FMT>(p, row, col, atomicExch(wsl + (int64_t)rr * MMA_BM + colt, 0) - p.corr[row]);
                    }
                    __syncwarp();
                    if (lane == 0) p.tickets[slot * 4 + q] = 0u;
                }
            }
            u += n;
            kb0 = 0;
            ++t;
            if (++rt == p.RT) { rt = 0; ++ct; }
        }
    }
    // warp 3 and the idle lanes fall through
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        __syncwarp();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(p.tmem_cols) : "memory");
    }
}

// per-row bias correction of the biased codes: 3.5-bit 8*sum(a, even k) + 4*sum(a, odd k),
// INT4 8*sum(a); one CTA per row
template <int FMT>
__global__ void rowcorr_kernel(const int8_t *__restrict__ x, int64_t sx_row, int32_t K, int32_t M,
                               int32_t *__restrict__ corr) {
    pdl_trigger();
    pdl_wait();
    const int row = blockIdx.x;
    if (row >= M) return;
    const int8_t *xr = x + row * sx_row;
    const uint32_t wts = (FMT == Q35_FMT_3P5BIT) ? 0x04080408u : 0x08080808u;
    int acc = 0;
    const int K4 = K & ~3;
    for (int k = 4 * threadIdx.x; k < K4; k += 4 * blockDim.x) {
        const uint32_t w = *reinterpret_cast<const uint32_t *>(xr + k);
        int d;
        asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(w), "r"(wts), "r"(acc));
        acc = d;
    }
    for (int k = K4 + threadIdx.x; k < K; k += blockDim.x)
        acc += (int)xr[k] * ((FMT == Q35_FMT_3P5BIT && (k & 1)) ? 4 : 8);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    __shared__ int part[32];
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x < 32) {
        int v = (threadIdx.x < (blockDim.x >> 5)) ? part[threadIdx.x] : 0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (threadIdx.x == 0) corr[row] = v;
    }
}

// dst[c * ld + r] = src[r][c] for a rows x cols int8 matrix (column-major activations to
// the row-major layout, rows ld bytes apart, that the tensor-core path reads through TMA)
__global__ void transpose_i8_kernel(const int8_t *__restrict__ src, int8_t *__restrict__ dst, int32_t rows,
                                    int32_t cols, int64_t ld) {
    __shared__ int8_t t[32][33];
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int r = r0 + i, c = c0 + threadIdx.x;
        if (r < rows && c < cols) t[i][threadIdx.x] = src[(int64_t)r * cols + c];
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int c = c0 + i, r = r0 + threadIdx.x;
        if (r < rows && c < cols) dst[(int64_t)c * ld + r] = t[threadIdx.x][i];
    }
}

int launch_transpose_i8(const int8_t *src, int8_t *dst, int32_t rows, int32_t cols, int64_t ld, cudaStream_t s) {
    const dim3 grid((unsigned)ceil_div(cols, 32), (unsigned)ceil_div(rows, 32));
    if (grid.y > 65535u) return set_error(Q35_ERR_INVALID, "transpose: too many rows");
    transpose_i8_kernel<<<grid, dim3(32, 8), 0, s>>>(src, dst, rows, cols, ld);
    Q35_CUDA_TRY(cudaGetLastError());
    return Q35_OK;
}

// ---- host side -------------------------------------------------------------------------
static int sm_count_of(int dev) {
    static int cached[64] = {0};
    if (dev < 0 || dev >= 64) return 148;
    if (!cached[dev]) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
        cached[dev] = v;
    }
    return cached[dev];
}

static int mma_bn(int32_t M) { return (int)min64(MMA_BN_MAX, round_up(M, 16)); }

struct MmaPlan {
    int BN, RT, CT, S, SB, P, grid, dual;
    int64_t per, work;
    uint32_t tmem_cols, a_col0;
    size_t off_b, off_pk, off_bar, smem;
};

static MmaPlan plan_mma(const Weights &w, int32_t M, int sms) {
    MmaPlan pl{};
    pl.BN = mma_bn(M);
    pl.RT = (int)ceil_div(M, pl.BN);
    pl.CT = (int)ceil_div(w.CG, 4);
    pl.work = (int64_t)pl.RT * pl.CT * w.KB;
    int64_t grid = min64(sms, pl.work);
    pl.per = ceil_div(pl.work, grid);
    pl.grid = (int)ceil_div(pl.work, pl.per);
    // tensor memory: accumulators [0, 2*BN) (two MMA issuers where they fit: [0, 4*BN)),
    // A stages from a_col0, 64 columns each
    pl.S = 4;
    pl.dual = 4 * pl.BN + 64 * pl.S <= 512 ? 1 : 0;
    pl.a_col0 = (uint32_t)((pl.dual ? 4 : 2) * pl.BN);
    pl.tmem_cols = 512;
    // shared memory: the activation ring (BN x 256 bytes a stage, 64-96 KB deep, 4 to 16
    // stages) and the packed-weight ring, which takes what is left (at most 12 stages);
    // that also keeps the CTA alone on its SM (it holds all of tensor memory)
    const size_t b_stage = (size_t)pl.BN * 256;
    const size_t pk_stage = 4 * w.tile_bytes;
    const size_t budget = 227 * 1024 - 1024 - 512;   // alignment slack, barriers
    pl.SB = (int)std::max<size_t>(4, std::min<size_t>(16, (pl.BN <= 16 ? 64 * 1024 : 96 * 1024) / b_stage));
    pl.P = (int)std::min<size_t>(12, (budget - (size_t)pl.SB * b_stage) / pk_stage);
    pl.off_b = 0;
    pl.off_pk = (size_t)pl.SB * b_stage;
    pl.off_bar = round_up((int64_t)(pl.off_pk + (size_t)pl.P * pk_stage), 8);
    pl.smem = 1024 + pl.off_bar + 8 * (2 * pl.P + 2 * pl.S + 2 * pl.SB + 5) + 16;
    return pl;
}

size_t mma_workspace_acc_elems(const Weights &w, int32_t M, int dev) {
    const MmaPlan pl = plan_mma(w, M, sm_count_of(dev));
    return (size_t)pl.grid * pl.BN * MMA_BM;
}
size_t mma_workspace_tickets(const Weights &w, int32_t M, int dev) {
    return (size_t)plan_mma(w, M, sm_count_of(dev)).grid * 4;
}

bool mma_supported(const Weights &w, const GemvArgs &a) {
    return a.M >= 1 && a.sx_k == 1 && a.sx_row >= w.K && (a.sx_row % 16) == 0 &&
           (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 && w.K >= 2 && w.K <= GEMM_MAX_K;
}

int launch_mma(const Weights &w, const GemvArgs &a, Workspace &ws, cudaStream_t s) {
    if (!mma_supported(w, a)) return set_error(Q35_ERR_INVALID, "mma: activations must be row-major, 16-byte aligned rows");
    const int dev = w.device;
    if (dev < 0 || dev >= 64) return set_error(Q35_ERR_INVALID, "mma: device ordinal out of range");
    const MmaPlan pl = plan_mma(w, a.M, sm_count_of(dev));
    if (!ws.acc || !ws.tickets || !ws.err || !ws.corr || ws.acc_elems < (size_t)pl.grid * pl.BN * MMA_BM ||
        ws.n_tickets < (size_t)pl.grid * 4 || ws.corr_elems < (size_t)a.M)
        return set_error(Q35_ERR_STATE, "mma: workspace too small");

    // the driver entry point is looked up through the runtime, so the library loads on
    // hosts without a driver (the build and CPU checks)
    using EncodeFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
    static EncodeFn encode = nullptr;
    if (!encode) {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
            return set_error(Q35_ERR_CUDA, "mma: cuTensorMapEncodeTiled not available");
        encode = reinterpret_cast<EncodeFn>(fn);
    }
    CUtensorMap map;
    const cuuint64_t dims[2] = {(cuuint64_t)w.K, (cuuint64_t)a.M};
    const cuuint64_t strides[1] = {(cuuint64_t)a.sx_row};
    const cuuint32_t box[2] = {128u, (cuuint32_t)pl.BN};
    const cuuint32_t estr[2] = {1u, 1u};
    CUresult cr = encode(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t *>(a.x), dims,
                                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return set_error(Q35_ERR_CUDA, "mma: cuTensorMapEncodeTiled failed");

    MmaParams p;
    p.tiles = w.tiles; p.scales = w.scales; p.offsets = w.offsets;
    p.KB = w.KB; p.CG = w.CG; p.N = w.N; p.K = w.K; p.M = a.M;
    p.BN = pl.BN; p.RT = pl.RT; p.CT = pl.CT; p.per = pl.per; p.work = pl.work;
    p.S = pl.S; p.SB = pl.SB; p.P = pl.P;
    p.tile_bytes = (uint32_t)w.tile_bytes;
    p.tmem_cols = pl.tmem_cols;
    p.C = a.C; p.y = a.y; p.res = a.res; p.so_row = a.so_row; p.so_col = a.so_col;
    p.corr = ws.corr; p.ws = ws.acc; p.tickets = ws.tickets; p.err = ws.err;
    p.off_b = (uint32_t)pl.off_b; p.off_pk = (uint32_t)pl.off_pk; p.off_bar = (uint32_t)pl.off_bar;
    p.a_col0 = pl.a_col0;
    p.dual = pl.dual;

    const bool f35 = w.format == Q35_FMT_3P5BIT;
    static bool configured[64][4] = {};
    auto kern = f35 ? (pl.dual ? mma_kernel<Q35_FMT_3P5BIT, true> : mma_kernel<Q35_FMT_3P5BIT, false>)
                    : (pl.dual ? mma_kernel<Q35_FMT_INT4, true> : mma_kernel<Q35_FMT_INT4, false>);
    const int ki = (f35 ? 0 : 2) + (pl.dual ? 1 : 0);
    if (!configured[dev][ki]) {
        int optin = 0;
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
        if (e != cudaSuccess) return set_error(Q35_ERR_CUDA, std::string("mma: shared memory ") + cudaGetErrorString(e));
        configured[dev][ki] = true;
    }

    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    // row corrections
    {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)a.M);
        cfg.blockDim = dim3(256);
        cfg.stream = s;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        auto ck = f35 ? rowcorr_kernel<Q35_FMT_3P5BIT> : rowcorr_kernel<Q35_FMT_INT4>;
        Q35_CUDA_TRY(cudaLaunchKernelEx(&cfg, ck, a.x, (int64_t)a.sx_row, (int32_t)w.K, (int32_t)a.M, ws.corr));
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)pl.grid);
    cfg.blockDim = dim3(MMA_THREADS);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    Q35_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, p, map));
    return Q35_OK;
}

}  // namespace q35
