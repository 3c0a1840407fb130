// tiled.cuh - the tiled expert layout and its one-time prepack kernel.
//
// Vault layout (shatter_moe.py:627-674): per matrix, row-major nibbles then
// row-major scales (then biases for AFFINE-Q4). Reading 16 rows of it needs
// one copy per row (1 KB or 384 B), and 1-D bulk copies that small run far
// below the HBM roofline on B200 (measured: 384 B -> 1.9 TB/s, >= 2 KB ->
// 5.5 TB/s over 148 SMs). The tiled layout makes each piece of work of the
// layer kernel (moe_layer.cuh) one contiguous block of a few tens of KB:
//
//   expert = [A unit 0 .. d_ff/16-1][B tile 0 .. d_model/16-1]
//   A unit u (hidden rows 16u..16u+15 of gate and up) = nchunk chunks,
//     chunk c (64-groups c*Gc .. c*Gc+Gc-1 of the input dimension) =
//       [gate frag][up frag][gate sb][up sb]
//   B tile o (output rows 16o..16o+15 of down, all d_ff columns) =
//       [codes: d_ff/64 groups x 512 B, the frag order below][sb: d_ff/64 groups x 16 rows]
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
// B codes: per 64-group 512 B in the A-fragment order of the integer MMA
//   m16n8k16 (u8), one MMA per 16-column unit u of the group: lane L = 4g + c
//   holds 16 B = words {row g, units 0-1}, {row g+8, units 0-1}, {row g,
//   units 2-3}, {row g+8, units 2-3}; byte b of a word holds the code of
//   column 16u + 4c + b of the even unit in its low nibble and of the odd unit
//   in its high nibble, so one mask per register gives q (even unit) or 16q
//   (odd unit).
// Byte count equals the vault layout's.
#pragma once
#include "smoe_common.cuh"

namespace smoe {

struct TiledGeom {
    uint32_t d, dff, G, Gd, e;      // dims, 64-groups of d and of d_ff, bytes per sb entry
    uint32_t nchunk, Gc;            // chunks per A unit, groups per chunk
    uint32_t fragC, sbC, chunk;     // one gate/up frag of a chunk, one sb block, whole chunk
    uint32_t aunit;                 // A unit bytes (nchunk chunks)
    uint32_t bcodes, btile;         // B tile codes, whole B tile
    uint64_t expert;
    __host__ __device__ bool init(int fmt, uint32_t d_, uint32_t dff_) {
        d = d_; dff = dff_; G = d / 64; Gd = dff / 64;
        e = (fmt == 1) ? 4 : 2;
        nchunk = (G + 31) / 32;
        Gc = nchunk ? G / nchunk : 0;
        fragC = Gc * 512; sbC = 16 * Gc * e;
        chunk = 2 * fragC + 2 * sbC;
        aunit = nchunk * chunk;
        bcodes = (dff / 16) * 128;
        btile = bcodes + Gd * 16 * e;
        expert = uint64_t(dff / 16) * aunit + uint64_t(d / 16) * btile;
        return d % 64 == 0 && dff % 64 == 0 && d > 0 && dff > 0 && G % nchunk == 0;
    }
    __host__ __device__ uint64_t chunk_off(uint32_t u, uint32_t c) const { return uint64_t(u) * aunit + uint64_t(c) * chunk; }
    __host__ __device__ uint64_t btile_off(uint32_t o) const { return uint64_t(dff / 16) * aunit + uint64_t(o) * btile; }
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

// grid (d_ff/16 + d_model/16, n_experts), 256 threads
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
    } else {
        const uint32_t o = blk - t.dff / 16;                // B tile: output rows 16o..16o+15
        uint8_t* p = dexp + t.btile_off(o);
        uint4* codes = reinterpret_cast<uint4*>(p);
        const uint8_t* dn = NIB(2);
        for (uint32_t i = threadIdx.x; i < t.Gd * 32; i += blockDim.x) {
            const uint32_t gi = i >> 5, L = i & 31, g = L >> 2, c = L & 3;
            uint32_t w[4];
            for (int q = 0; q < 4; ++q) {                         // (row g / g+8) x (units 0-1 / 2-3)
                const uint8_t* row = dn + size_t(o * 16 + g + 8 * (q & 1)) * (t.dff / 2);
                const uint32_t u0 = 2 * (q >> 1);
                uint32_t v = 0;
                for (uint32_t b = 0; b < 4; ++b) {
                    const uint32_t col = gi * 64 + 4 * c + b;
                    v |= (nib_at(row, col + 16 * u0) | (nib_at(row, col + 16 * (u0 + 1)) << 4)) << (8 * b);
                }
                w[q] = v;
            }
            codes[i] = make_uint4(w[0], w[1], w[2], w[3]);
        }
        uint8_t* sb = p + t.bcodes;
        for (uint32_t i = threadIdx.x; i < t.Gd * 16; i += blockDim.x) {
            const uint32_t grp = i >> 4, r = i & 15;
            put_sb(sb, i, 2, size_t(o * 16 + r) * t.Gd + grp);
        }
    }
}

}  // namespace smoe
