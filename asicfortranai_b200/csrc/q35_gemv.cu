// q35_gemv.cu -- decode GEMV / skinny GEMM on CUDA cores (dp4a), exact int32.
//
// Computes, for the reference kernels matmul_3p5bit_awq (matmul_3p5bit_dynamic.f90:42-64)
// and matmul_int4_awq (matmul_int4_groq.f90:117-137):
//   C(i,j) = sum_k A(i,k) * code(k,j)          (int32, exact)
//   y(i,j) = (float(C) + offset_j) * scale_j   (3.5-bit, :80)   or  float(C) * scale_j (INT4)
//
// Work split: a CTA of 8 warps owns 8 column groups (256 columns) and a range of
// k-blocks; every lane owns one column.  The CTA stages its activation rows for that
// k range in shared memory in the even/odd image order, so each extracted weight word
// is multiplied by one broadcast shared-memory word with dp4a.  Weights are streamed
// with 16-byte non-caching loads, two k-blocks in flight per warp.
//
// Split-K: when a column block is split over S CTAs, each CTA adds its exact partial
// sums into an int32 workspace with atomicAdd (integer addition is order-free, so the
// result is bit-identical to a single pass), then takes a ticket; the last CTA of the
// column block reads the totals back with atomicExch(.., 0), which also leaves the
// workspace zero for the next call, runs the dequant epilogue and resets the ticket.
#include "q35_internal.cuh"

namespace q35 {

constexpr int GEMV_WARPS = 8;
constexpr int GEMV_THREADS = GEMV_WARPS * 32;
constexpr int GEMV_SMEM_MAX = 46 * 1024;   // dynamic, below the 48 KB default with static smem

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
    int32_t R, S;            // k-blocks per split, number of splits
    int32_t *ws_acc;         // [M][CG*32], zero between calls
    uint32_t *tickets;       // [row chunks][gridDim.x], zero between calls
};

__device__ __forceinline__ int dp4a(uint32_t a, uint32_t b, int c) {
    return __dp4a((int)a, (int)b, c);   // weight bytes are 0..15: same value as s8
}

__device__ __forceinline__ uint4 ld_stream(const uint4 *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// dot of one 3.5-bit tile record (28 words) with one activation image (64 words)
__device__ __forceinline__ int dot35(const uint32_t (&W)[32], const uint32_t *img, int acc) {
    const uint4 *E4 = reinterpret_cast<const uint4 *>(img);
    const uint4 *O4 = reinterpret_cast<const uint4 *>(img + 32);
#pragma unroll
    for (int q = 0; q < 8; ++q) {                       // nibble plane: 2 words per uint4
        uint4 e = E4[q];
        uint32_t w0 = W[2 * q], w1 = W[2 * q + 1];
        acc = dp4a(w0 & 0x0F0F0F0Fu, e.x, acc);
        acc = dp4a((w0 >> 4) & 0x0F0F0F0Fu, e.y, acc);
        acc = dp4a(w1 & 0x0F0F0F0Fu, e.z, acc);
        acc = dp4a((w1 >> 4) & 0x0F0F0F0Fu, e.w, acc);
    }
#pragma unroll
    for (int w = 0; w < 8; ++w) {                       // 2-bit plane: O words 4w..4w+3
        uint4 o = O4[w];
        uint32_t v = W[16 + w];
        acc = dp4a(v & 0x03030303u, o.x, acc);
        acc = dp4a((v >> 2) & 0x03030303u, o.y, acc);
        acc = dp4a((v >> 4) & 0x03030303u, o.z, acc);
        acc = dp4a((v >> 6) & 0x03030303u, o.w, acc);
    }
#pragma unroll
    for (int w = 0; w < 4; ++w) {                       // 1-bit plane (weight 4): O words 8w..8w+7
        uint4 o0 = O4[2 * w], o1 = O4[2 * w + 1];
        uint32_t v = W[24 + w];
        acc = dp4a((v << 2) & 0x04040404u, o0.x, acc);
        acc = dp4a((v << 1) & 0x04040404u, o0.y, acc);
        acc = dp4a(v & 0x04040404u, o0.z, acc);
        acc = dp4a((v >> 1) & 0x04040404u, o0.w, acc);
        acc = dp4a((v >> 2) & 0x04040404u, o1.x, acc);
        acc = dp4a((v >> 3) & 0x04040404u, o1.y, acc);
        acc = dp4a((v >> 4) & 0x04040404u, o1.z, acc);
        acc = dp4a((v >> 5) & 0x04040404u, o1.w, acc);
    }
    return acc;
}

// dot of one INT4 tile record (32 words) with one activation image
__device__ __forceinline__ int dot4(const uint32_t (&W)[32], const uint32_t *img, int acc) {
    const uint4 *I4 = reinterpret_cast<const uint4 *>(img);
#pragma unroll
    for (int q = 0; q < 16; ++q) {
        uint4 e = I4[q];
        uint32_t w0 = W[2 * q], w1 = W[2 * q + 1];
        acc = dp4a(w0 & 0x0F0F0F0Fu, e.x, acc);
        acc = dp4a((w0 >> 4) & 0x0F0F0F0Fu, e.y, acc);
        acc = dp4a(w1 & 0x0F0F0F0Fu, e.z, acc);
        acc = dp4a((w1 >> 4) & 0x0F0F0F0Fu, e.w, acc);
    }
    return acc;
}

template <int FMT>
__device__ __forceinline__ void load_tile(const uint4 *p, uint32_t (&W)[32]) {
    constexpr int NC = (FMT == Q35_FMT_3P5BIT) ? 7 : 8;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
        uint4 v = ld_stream(p + c * 32);
        W[4 * c] = v.x; W[4 * c + 1] = v.y; W[4 * c + 2] = v.z; W[4 * c + 3] = v.w;
    }
}

__device__ __forceinline__ float dequant(int FMT, int32_t c, const float *scales,
                                         const float *offsets, int64_t j) {
    float f = __int2float_rn(c);
    if (FMT == Q35_FMT_3P5BIT) return __fmul_rn(__fadd_rn(f, offsets[j]), scales[j]);
    return __fmul_rn(f, scales[j]);
}

template <int FMT, int MT>
__global__ void __launch_bounds__(GEMV_THREADS)
gemv_kernel(const GemvParams p) {
    extern __shared__ __align__(16) uint32_t smem[];
    __shared__ int32_t s_corr[MT];
    __shared__ int s_last;
    constexpr int TU4 = ((FMT == Q35_FMT_3P5BIT) ? 7 : 8) * 32;   // uint4 per tile

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int cg = blockIdx.x * GEMV_WARPS + warp;
    const bool active = cg < p.CG;
    const int kb0 = blockIdx.y * p.R;
    const int nkb = min(p.KB - kb0, p.R);
    const int64_t j = (int64_t)cg * 32 + lane;
    const int64_t Np = (int64_t)p.CG * 32;
    const int nchunks = (p.M + MT - 1) / MT;
    uint8_t *img8 = reinterpret_cast<uint8_t *>(smem);

    for (int chunk = 0; chunk < nchunks; ++chunk) {
        const int r0 = chunk * MT;
        // ---- stage activations rows r0..r0+MT-1, k-blocks kb0..kb0+nkb-1 ----
        if (tid < MT) s_corr[tid] = 0;
        __syncthreads();
        const int per_row = nkb * KBLK;
#pragma unroll 1
        for (int r = 0; r < MT; ++r) {
            const int row = r0 + r;
            int corr = 0;
            for (int e = tid; e < per_row; e += GEMV_THREADS) {
                const int kbl = e / KBLK, byte = e % KBLK;
                const int word = byte >> 2, b = byte & 3;
                const bool odd = word >= 32;
                const int64_t pair = (int64_t)(kb0 + kbl) * PAIRS + 4 * (word & 31) + b;
                const int64_t k = 2 * pair + (odd ? 1 : 0);
                int v = 0;
                if (row < p.M && k < p.K) v = p.x[row * p.sx_row + k * p.sx_k];
                img8[(r * p.R + kbl) * KBLK + byte] = (uint8_t)(int8_t)v;
                corr += (FMT == Q35_FMT_3P5BIT) ? (odd ? 4 : 8) * v : 8 * v;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) corr += __shfl_xor_sync(0xffffffffu, corr, o);
            if (lane == 0 && corr != 0) atomicAdd(&s_corr[r], corr);
        }
        __syncthreads();

        // ---- stream the weight tiles ----
        int32_t acc[MT];
#pragma unroll
        for (int r = 0; r < MT; ++r) acc[r] = 0;
        if (active && nkb > 0) {
            const uint4 *tp = p.tiles + ((size_t)cg * p.KB + kb0) * TU4 + lane;
            uint32_t cur[32], nxt[32];
            load_tile<FMT>(tp, cur);
#pragma unroll 1
            for (int kbl = 0; kbl < nkb; ++kbl) {
                if (kbl + 1 < nkb) load_tile<FMT>(tp + (size_t)(kbl + 1) * TU4, nxt);
#pragma unroll
                for (int r = 0; r < MT; ++r) {
                    const uint32_t *img = smem + (r * p.R + kbl) * (KBLK / 4);
                    acc[r] = (FMT == Q35_FMT_3P5BIT) ? dot35(cur, img, acc[r]) : dot4(cur, img, acc[r]);
                }
#pragma unroll
                for (int t = 0; t < 32; ++t) cur[t] = nxt[t];
            }
        }
#pragma unroll
        for (int r = 0; r < MT; ++r) acc[r] -= s_corr[r];

        // ---- epilogue ----
        if (p.S == 1) {
            if (active && j < p.N) {
#pragma unroll
                for (int r = 0; r < MT; ++r) {
                    const int row = r0 + r;
                    if (row < p.M) {
                        const int64_t o = row * p.so_row + j * p.so_col;
                        if (p.C) p.C[o] = acc[r];
                        if (p.y) p.y[o] = dequant(FMT, acc[r], p.scales, p.offsets, j);
                    }
                }
            }
        } else {
            if (active && j < p.N) {
#pragma unroll
                for (int r = 0; r < MT; ++r) {
                    const int row = r0 + r;
                    if (row < p.M && acc[r] != 0) atomicAdd(&p.ws_acc[row * Np + j], acc[r]);
                }
            }
            __threadfence();
            __syncthreads();
            if (tid == 0) {
                uint32_t *t = &p.tickets[chunk * gridDim.x + blockIdx.x];
                s_last = (atomicAdd(t, 1u) == (uint32_t)(p.S - 1));
            }
            __syncthreads();
            if (s_last) {
                __threadfence();
                if (active && j < p.N) {
#pragma unroll
                    for (int r = 0; r < MT; ++r) {
                        const int row = r0 + r;
                        if (row < p.M) {
                            const int32_t v = atomicExch(&p.ws_acc[row * Np + j], 0);
                            const int64_t o = row * p.so_row + j * p.so_col;
                            if (p.C) p.C[o] = v;
                            if (p.y) p.y[o] = dequant(FMT, v, p.scales, p.offsets, j);
                        }
                    }
                }
                if (tid == 0) p.tickets[chunk * gridDim.x + blockIdx.x] = 0u;
            }
        }
        __syncthreads();   // the image is rewritten by the next row chunk
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

static int pick_mt(int32_t M) { return M <= 1 ? 1 : (M <= 2 ? 2 : (M <= 4 ? 4 : 8)); }

struct Plan { int MT, nbx, R, S; size_t smem; };

static Plan make_plan(const Weights &w, int32_t M) {
    Plan pl;
    pl.MT = pick_mt(M);
    pl.nbx = (int)ceil_div(w.CG, GEMV_WARPS);
    const int target = 2 * sm_count(w.device);
    int S = (int)std::min<int64_t>(std::max<int64_t>(ceil_div(target, pl.nbx), 1), w.KB);
    int R = (int)ceil_div(w.KB, S);
    const int rmax = GEMV_SMEM_MAX / (pl.MT * KBLK);
    if (R > rmax) R = rmax;
    S = (int)ceil_div(w.KB, R);
    pl.R = R;
    pl.S = S;
    pl.smem = (size_t)pl.MT * R * KBLK;
    return pl;
}

size_t gemv_workspace_acc_elems(const Weights &w, int32_t M) {
    Plan pl = make_plan(w, M);
    return pl.S > 1 ? (size_t)M * w.CG * 32 : 0;
}

size_t gemv_workspace_tickets(const Weights &w) {
    return (size_t)ceil_div(w.CG, GEMV_WARPS) * 8;   // up to 8 row chunks (M <= 64)
}

template <int FMT, int MT>
static void launch_t(const GemvParams &p, const Plan &pl, cudaStream_t s) {
    dim3 grid(pl.nbx, pl.S);
    gemv_kernel<FMT, MT><<<grid, GEMV_THREADS, pl.smem, s>>>(p);
}

int launch_gemv(const Weights &w, const GemvArgs &a, Workspace &ws, cudaStream_t s) {
    if (a.M <= 0 || a.M > 64) return set_error(Q35_ERR_INVALID, "gemv: M must be in [1,64]");
    Plan pl = make_plan(w, a.M);
    GemvParams p;
    p.tiles = reinterpret_cast<const uint4 *>(w.tiles);
    p.scales = w.scales;
    p.offsets = w.offsets;
    p.KB = w.KB; p.CG = w.CG; p.N = w.N; p.K = w.K;
    p.x = a.x; p.sx_row = a.sx_row; p.sx_k = a.sx_k; p.M = a.M;
    p.C = a.C; p.y = a.y; p.so_row = a.so_row; p.so_col = a.so_col;
    p.R = pl.R; p.S = pl.S;
    p.ws_acc = ws.acc;
    p.tickets = ws.tickets;
    if (pl.S > 1) {
        if (!ws.acc || ws.acc_elems < (size_t)a.M * w.CG * 32 || !ws.tickets ||
            ws.n_tickets < gemv_workspace_tickets(w))
            return set_error(Q35_ERR_STATE, "gemv: split-K workspace too small");
    }
    const bool f35 = w.format == Q35_FMT_3P5BIT;
    switch (pl.MT) {
        case 1: f35 ? launch_t<Q35_FMT_3P5BIT, 1>(p, pl, s) : launch_t<Q35_FMT_INT4, 1>(p, pl, s); break;
        case 2: f35 ? launch_t<Q35_FMT_3P5BIT, 2>(p, pl, s) : launch_t<Q35_FMT_INT4, 2>(p, pl, s); break;
        case 4: f35 ? launch_t<Q35_FMT_3P5BIT, 4>(p, pl, s) : launch_t<Q35_FMT_INT4, 4>(p, pl, s); break;
        default: f35 ? launch_t<Q35_FMT_3P5BIT, 8>(p, pl, s) : launch_t<Q35_FMT_INT4, 8>(p, pl, s); break;
    }
    Q35_CUDA_TRY(cudaGetLastError());
    return Q35_OK;
}

}  // namespace q35
