// tiled.cuh - the tiled expert layout and its one-time prepack kernel.
//
// Vault layout (shatter_moe.py:627-674): per matrix, row-major nibbles then
// row-major scales (then biases for AFFINE-Q4). Reading 16 rows of it needs
// one copy per row (1 KB or 384 B), and 1-D bulk copies that small run far
// below the HBM roofline on B200 (measured: 384 B -> 1.9 TB/s, >= 2 KB ->
// 5.5 TB/s over 148 SMs). The tiled layout makes each piece of work of the
// layer kernel (moe_layer.cuh) one contiguous block of a few tens of KB:
//
//   expert = [A unit 0 .. d_ff/16-1][D unit 0 .. d_ff/16-1][S group 0 .. d_ff/64-1]
//   A unit u (hidden rows 16u..16u+15 of gate and up) = nchunk chunks,
//     chunk c (64-groups c*Gc .. c*Gc+Gc-1 of the input dimension) =
//       [gate frag][up frag][gate sb][up sb]
//   D unit u (columns 16u..16u+15 of down - the ones hidden unit u feeds -
//     all d_model rows) = d_model/64 blocks of 512 B, the frag order below
//   S group j (down's scales of d_ff group j, all d_model rows, row order)
//
// nchunk = ceil(G / 32) (G = d_model/64 groups), Gc = G / nchunk: chunks of
// at most 32 groups (36 KB) so that a few of them fit in shared memory.
// gate/up frag: the 16 x (64 Gc) nibble tile in the A-fragment order of the
//   integer MMA m16n8k32 (u8): per 64-group 512 B, lane L = 4g + c holding
//   16 B at L*16 = words c and c+4 (bytes 4c..4c+3 and 16+4c..16+4c+3 of the
//   row's 32-byte group segment) of rows g and g+8, in the order
//   [row g word c][row g+8 word c][row g word c+4][row g+8 word c+4], which
//   is registers a0..a3. Byte b of a segment holds columns 2b (low nibble)
//   and 2b+1 (high nibble), so the low and high nibbles of the same registers
//   feed two MMAs over the even and the odd columns. A warp's fragment loads
//   are consecutive in shared memory (no bank conflicts).
// sb: per-group scales transposed to [group][16 rows]; AFFINE-Q4 packs
//   (scale, bias) into one 32-bit word (scale in the low half), SMOE-Q4 holds
//   the 16-bit scale alone.
// D block b (rows 64b..64b+63 of down, the unit's 16 columns): four row
//   tiles of 16 rows in the A-fragment order of the integer MMA m16n8k16
//   (u8), two tiles per byte: lane L = 4g + c holds 16 B = words {tiles 0-1,
//   row g}, {tiles 0-1, row g+8}, {tiles 2-3, row g}, {tiles 2-3, row g+8}
//   (row r of tile q = row 64b + 16q + r); byte j of a word holds column
//   16u + 4c + j of the even tile in its low nibble and of the odd tile in
//   its high nibble.
// Byte count equals the vault layout's.
#pragma once
#include "smoe_common.cuh"

namespace smoe {

struct TiledGeom {
    uint32_t d, dff, G, Gd, e;      // dims, 64-groups of d and of d_ff, bytes per sb entry
    uint32_t nchunk, Gc;            // chunks per A unit, groups per chunk
    uint32_t fragC, sbC, chunk;     // one gate/up frag of a chunk, one sb block, whole chunk
    uint32_t aunit;                 // A unit bytes (nchunk chunks)
    uint32_t dunit, sgrp;           // one D unit, one S group
    uint64_t expert;
    __host__ __device__ bool init(int fmt, uint32_t d_, uint32_t dff_) {
        d = d_; dff = dff_; G = d / 64; Gd = dff / 64;
        e = (fmt == 1) ? 4 : 2;
        nchunk = (G + 31) / 32;
        Gc = nchunk ? G / nchunk : 0;
        fragC = Gc * 512; sbC = 16 * Gc * e;
        chunk = 2 * fragC + 2 * sbC;
        aunit = nchunk * chunk;
        dunit = d * 8;
        sgrp = d * e;
        expert = uint64_t(dff / 16) * (aunit + dunit) + uint64_t(Gd) * sgrp;
        return d % 64 == 0 && dff % 64 == 0 && d > 0 && dff > 0 && G % nchunk == 0;
    }
    __host__ __device__ uint64_t chunk_off(uint32_t u, uint32_t c) const { return uint64_t(u) * aunit + uint64_t(c) * chunk; }
    __host__ __device__ uint64_t dunit_off(uint32_t u) const { return uint64_t(dff / 16) * aunit + uint64_t(u) * dunit; }
    __host__ __device__ uint64_t sgrp_off(uint32_t j) const {
        return uint64_t(dff / 16) * (aunit + dunit) + uint64_t(j) * sgrp;
    }
};

struct PrepackArgs {
    const uint8_t* src;             // vault-layout arena
    uint64_t src_stride;
    uint64_t off[9];
    uint8_t* dst;                   // tiled arena
    uint64_t dst_stride;
    int fmt;
    TiledGeom tg;
};

SMOE_DEVINL uint32_t nib_at(const uint8_t* rowp, uint32_t col) {
    return (rowp[col >> 1] >> ((col & 1) * 4)) & 0xfu;
}

// grid (2 * d_ff/16 + d_ff/64, n_experts), 256 threads
__global__ void k_prepack(PrepackArgs a) {
    const TiledGeom& t = a.tg;
    const uint32_t e = blockIdx.y, blk = blockIdx.x;
    const uint8_t* s = a.src + uint64_t(e) * a.src_stride;
    uint8_t* dexp = a.dst + uint64_t(e) * a.dst_stride;
    auto NIB = [&](int m) { return s + a.off[3 * m]; };
    auto SC = [&](int m) { return reinterpret_cast<const uint16_t*>(s + a.off[3 * m + 1]); };
    auto BI = [&](int m) { return reinterpret_cast<const uint16_t*>(s + a.off[3 * m + 2]); };
    const bool aff = a.fmt == 1;
    auto put_sb = [&](uint8_t* sb, uint32_t i, int m, size_t idx) {
        const uint16_t sc = SC(m)[idx];
        if (aff) reinterpret_cast<uint32_t*>(sb)[i] = sc | (uint32_t(BI(m)[idx]) << 16);
        else reinterpret_cast<uint16_t*>(sb)[i] = sc;
    };
    if (blk < t.dff / 16) {
        const uint32_t u = blk, row0 = u * 16;
        for (uint32_t c = 0; c < t.nchunk; ++c) {
            uint8_t* p = dexp + t.chunk_off(u, c);
            for (int m = 0; m < 2; ++m) {                   // gate / up fragments
                const uint8_t* nib = NIB(m);
                uint4* frag = reinterpret_cast<uint4*>(p + m * t.fragC);
                for (uint32_t i = threadIdx.x; i < t.Gc * 32; i += blockDim.x) {
                    const uint32_t gl = i >> 5, lane = i & 31, g = lane >> 2, cc = lane & 3;
                    const uint32_t grp = c * t.Gc + gl;
                    const uint32_t* rg = reinterpret_cast<const uint32_t*>(nib + size_t(row0 + g) * (t.d / 2) + grp * 32);
                    const uint32_t* rh = reinterpret_cast<const uint32_t*>(nib + size_t(row0 + g + 8) * (t.d / 2) + grp * 32);
                    frag[i] = make_uint4(rg[cc], rh[cc], rg[cc + 4], rh[cc + 4]);
                }
                uint8_t* sb = p + 2 * t.fragC + m * t.sbC;
                for (uint32_t i = threadIdx.x; i < t.Gc * 16; i += blockDim.x) {
                    const uint32_t gl = i >> 4, r = i & 15;
                    put_sb(sb, i, m, size_t(row0 + r) * t.G + c * t.Gc + gl);
                }
            }
        }
    } else if (blk < 2 * (t.dff / 16)) {
        const uint32_t u = blk - t.dff / 16;                // D unit: down columns 16u..16u+15
        uint4* codes = reinterpret_cast<uint4*>(dexp + t.dunit_off(u));
        const uint8_t* dn = NIB(2);
        for (uint32_t i = threadIdx.x; i < (t.d / 64) * 32; i += blockDim.x) {
            const uint32_t b = i >> 5, L = i & 31, g = L >> 2, c = L & 3;
            uint32_t w[4];
            for (int q = 0; q < 4; ++q) {                   // (tiles 0-1 / 2-3) x (row g / g+8)
                const uint32_t tp = q >> 1, r = g + 8 * (q & 1);
                const uint8_t* lo = dn + size_t(64 * b + 16 * (2 * tp) + r) * (t.dff / 2);
                const uint8_t* hi = dn + size_t(64 * b + 16 * (2 * tp + 1) + r) * (t.dff / 2);
                uint32_t v = 0;
                for (uint32_t j = 0; j < 4; ++j) {
                    const uint32_t col = 16 * u + 4 * c + j;
                    v |= (nib_at(lo, col) | (nib_at(hi, col) << 4)) << (8 * j);
                }
                w[q] = v;
            }
            codes[i] = make_uint4(w[0], w[1], w[2], w[3]);
        }
    } else {
        const uint32_t j = blk - 2 * (t.dff / 16);          // S group j: down's scales, row order
        uint8_t* sb = dexp + t.sgrp_off(j);
        for (uint32_t r = threadIdx.x; r < t.d; r += blockDim.x) put_sb(sb, r, 2, size_t(r) * t.Gd + j);
    }
}

}  // namespace smoe
