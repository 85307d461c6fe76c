// q35_pack.cu -- builds the device streaming format from the reference's packed bytes
// (and back, for round-trip checks).  See q35_internal.cuh for the format.
#include "q35_internal.cuh"

namespace q35 {

// Decode of one reference byte, matmul_3p5bit_dynamic.f90:48-56 (raw7 = byte & 0x7F,
// n1 = raw7>>3 as 4-bit two's complement, n2 = raw7&7 as 3-bit two's complement);
// biased codes: b1 = n1+8 = (raw7>>3) ^ 8, b2 = n2+4 = (raw7&7) ^ 4.
__device__ __forceinline__ void decode35(uint8_t raw, uint32_t &b1, uint32_t &b2) {
    uint32_t r7 = raw & 0x7Fu;
    b1 = (r7 >> 3) ^ 8u;
    b2 = (r7 & 7u) ^ 4u;
}

// matmul_int4_groq.f90:126-133: low nibble -> even k, high nibble -> odd k.
__device__ __forceinline__ void decode4(uint8_t raw, uint32_t &be, uint32_t &bo) {
    be = (raw & 0xFu) ^ 8u;
    bo = ((raw >> 4) & 0xFu) ^ 8u;
}

// nibble plane word w from 128 biased 4-bit codes c[]: byte b = c[8w+b] | c[8w+4+b]<<4
__device__ __forceinline__ uint32_t nib_word(const uint8_t *c, int w) {
    uint32_t v = 0;
#pragma unroll
    for (int b = 0; b < 4; ++b) v |= (uint32_t)(c[8 * w + b] | (c[8 * w + 4 + b] << 4)) << (8 * b);
    return v;
}

// One thread per (column group, k-block, lane): reads the 128 reference bytes of its
// column for the k-block and writes its 7 (3.5-bit) or 8 (INT4) chunks.
template <int FMT>
__global__ void repack_kernel(const int8_t *__restrict__ ref, uint8_t *__restrict__ tiles,
                              int32_t K, int32_t N, int32_t KB, int32_t CG) {
    int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int64_t total = (int64_t)CG * KB * CGW;
    if (gid >= total) return;
    const int lane = (int)(gid % CGW);
    const int64_t tile = gid / CGW;            // = cg*KB + kb
    const int kb = (int)(tile % KB);
    const int cg = (int)(tile / KB);
    const int64_t j = (int64_t)cg * CGW + lane;
    const int64_t KH = K / 2;
    uint8_t e[PAIRS], o[PAIRS];
#pragma unroll 4
    for (int p = 0; p < PAIRS; ++p) {
        int64_t pg = (int64_t)kb * PAIRS + p;
        uint32_t a, b;
        if (j < N && pg < KH) {
            uint8_t raw = (uint8_t)ref[pg + KH * j];
            if (FMT == Q35_FMT_3P5BIT) decode35(raw, a, b); else decode4(raw, a, b);
        } else {
            a = 8u;
            b = (FMT == Q35_FMT_3P5BIT) ? 4u : 8u;   // codes that decode to 0
        }
        e[p] = (uint8_t)a;
        o[p] = (uint8_t)b;
    }
    uint32_t wds[32];
    int nwords;
    if (FMT == Q35_FMT_3P5BIT) {
        // 4 groups of 32 pairs; word i of group g, byte b: field of pair 32g+4i+b in bits
        // 0..6 and bit i of the field of pair 32g+28+b in bit 7
#pragma unroll
        for (int g = 0; g < 4; ++g) {
#pragma unroll
            for (int i = 0; i < 7; ++i) {
                uint32_t v = 0;
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const int pr = 32 * g + 4 * i + b, px = 32 * g + 28 + b;
                    const uint32_t f = (uint32_t)(o[pr] & 7u) | ((uint32_t)(e[pr] & 15u) << 3);
                    const uint32_t fx = (uint32_t)(o[px] & 7u) | ((uint32_t)(e[px] & 15u) << 3);
                    v |= (f | (((fx >> i) & 1u) << 7)) << (8 * b);
                }
                wds[7 * g + i] = v;
            }
        }
        nwords = 28;
    } else {
#pragma unroll
        for (int w = 0; w < 16; ++w) wds[w] = nib_word(e, w);
#pragma unroll
        for (int w = 0; w < 16; ++w) wds[16 + w] = nib_word(o, w);
        nwords = 32;
    }
    const size_t tb = (FMT == Q35_FMT_3P5BIT) ? TILE35 : TILE4;
    uint8_t *dst = tiles + (size_t)tile * tb + (size_t)lane * 16;
    for (int c = 0; c < nwords / 4; ++c) {
        uint4 v = make_uint4(wds[4 * c], wds[4 * c + 1], wds[4 * c + 2], wds[4 * c + 3]);
        *reinterpret_cast<uint4 *>(dst + (size_t)c * 512) = v;
    }
}

// Inverse of repack_kernel: rebuilds the reference bytes (the MSB, which the
// reference ignores, comes back as 0).
template <int FMT>
__global__ void unpack_kernel(const uint8_t *__restrict__ tiles, int8_t *__restrict__ ref,
                              int32_t K, int32_t N, int32_t KB, int32_t CG) {
    int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int64_t total = (int64_t)CG * KB * CGW;
    if (gid >= total) return;
    const int lane = (int)(gid % CGW);
    const int64_t tile = gid / CGW;
    const int kb = (int)(tile % KB);
    const int cg = (int)(tile / KB);
    const int64_t j = (int64_t)cg * CGW + lane;
    if (j >= N) return;
    const size_t tb = (FMT == Q35_FMT_3P5BIT) ? TILE35 : TILE4;
    const uint8_t *src = tiles + (size_t)tile * tb + (size_t)lane * 16;
    uint32_t wds[32];
    const int nwords = (FMT == Q35_FMT_3P5BIT) ? 28 : 32;
    for (int c = 0; c < nwords / 4; ++c) {
        uint4 v = *reinterpret_cast<const uint4 *>(src + (size_t)c * 512);
        wds[4 * c] = v.x; wds[4 * c + 1] = v.y; wds[4 * c + 2] = v.z; wds[4 * c + 3] = v.w;
    }
    const int64_t KH = K / 2;
    for (int p = 0; p < PAIRS; ++p) {
        int64_t pg = (int64_t)kb * PAIRS + p;
        if (pg >= KH) break;
        uint8_t out;
        if (FMT == Q35_FMT_3P5BIT) {
            const int g = p / 32, q = p % 32;
            uint32_t f;
            if (q < 28) {
                f = (wds[7 * g + q / 4] >> (8 * (q % 4))) & 0x7Fu;
            } else {
                f = 0;
                for (int i = 0; i < 7; ++i) f |= ((wds[7 * g + i] >> (8 * (q - 28) + 7)) & 1u) << i;
            }
            const uint32_t b2 = f & 7u, b1 = (f >> 3) & 15u;
            out = (uint8_t)((((b1 ^ 8u) & 0xFu) << 3) | ((b2 ^ 4u) & 7u));
        } else {
            const int w = p / 8, r = p % 8;
            const uint32_t be = (wds[w] >> (8 * (r % 4) + 4 * (r / 4))) & 0xFu;
            const uint32_t bo = (wds[16 + w] >> (8 * (r % 4) + 4 * (r / 4))) & 0xFu;
            out = (uint8_t)(((be ^ 8u) & 0xFu) | (((bo ^ 8u) & 0xFu) << 4));
        }
        ref[pg + KH * j] = (int8_t)out;
    }
}

int launch_repack(const Weights &w, const int8_t *d_ref, cudaStream_t s) {
    int64_t total = (int64_t)w.CG * w.KB * CGW;
    int threads = 128;
    int64_t blocks = ceil_div(total, threads);
    if (w.format == Q35_FMT_3P5BIT)
        repack_kernel<Q35_FMT_3P5BIT><<<(unsigned)blocks, threads, 0, s>>>(d_ref, w.tiles, w.K, w.N, w.KB, w.CG);
    else
        repack_kernel<Q35_FMT_INT4><<<(unsigned)blocks, threads, 0, s>>>(d_ref, w.tiles, w.K, w.N, w.KB, w.CG);
    Q35_CUDA_TRY(cudaGetLastError());
    return Q35_OK;
}

int launch_unpack_ref(const Weights &w, int8_t *d_ref, cudaStream_t s) {
    int64_t total = (int64_t)w.CG * w.KB * CGW;
    int threads = 128;
    int64_t blocks = ceil_div(total, threads);
    if (w.format == Q35_FMT_3P5BIT)
        unpack_kernel<Q35_FMT_3P5BIT><<<(unsigned)blocks, threads, 0, s>>>(w.tiles, d_ref, w.K, w.N, w.KB, w.CG);
    else
        unpack_kernel<Q35_FMT_INT4><<<(unsigned)blocks, threads, 0, s>>>(w.tiles, d_ref, w.K, w.N, w.KB, w.CG);
    Q35_CUDA_TRY(cudaGetLastError());
    return Q35_OK;
}

}  // namespace q35
