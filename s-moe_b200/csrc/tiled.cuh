// tiled.cuh - the tiled expert layout and its one-time prepack kernel.
//
// Vault layout (shatter_moe.py:627-674): per matrix, row-major nibbles then
// row-major scales (then biases for AFFINE-Q4). Reading 16 rows of it needs
// one copy per row (1 KB or 384 B), and 1-D bulk copies that small run far
// below the HBM roofline on B200 (measured: 384 B -> 1.9 TB/s, >= 2 KB ->
// 5.5 TB/s over 148 SMs). The tiled layout makes the fused kernel's unit of
// work - 16 hidden rows of one expert - one contiguous block:
//
//   expert = [unit 0 .. unit d_ff/16-1][down scales of group 0 .. d_ff/64-1]
//   unit u = [gate frag][up frag][gate sb][up sb]
//            [down slice: W_down[:, 16u .. 16u+15], fragment order]
//   group  = [down sc, d_model entries][down bias, d_model entries]
//
// gate/up frag: the 16 x d_model nibble tile in the A-fragment order of the
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
// down slice: per 16-row output tile, 32 words of 32 bits; word L (row
//   g = L/4, pair c = L%4) holds the codes of rows g and g+8 at columns 2c,
//   2c+1, 2c+8, 2c+9 of the slice in the bit order the kernel unpacks with
//   one mask per operand register (bits 0-3/16-19 row g cols 2c/2c+1, 4-7/
//   20-23 row g+8, 8-11/24-27 row g cols 2c+8/2c+9, 12-15/28-31 row g+8).
// Biases exist for AFFINE-Q4 only. Byte count equals the vault layout's.
#pragma once
#include "smoe_common.cuh"

namespace smoe {

struct TiledGeom {
    uint32_t d, dff, G, Gd;
    uint32_t fragA, sbA, gateup;    // bytes: one gate/up frag, one sb block, gate+up part of a unit
    uint32_t slice, unit;           // down slice bytes, whole unit bytes
    uint32_t dsc, dgroup;           // down scales of one group (per array), whole group block
    uint64_t expert;
    __host__ __device__ void init(int fmt, uint32_t d_, uint32_t dff_) {
        d = d_; dff = dff_; G = d / 64; Gd = dff / 64;
        const uint32_t nsb = (fmt == 1) ? 2 : 1;            // scale (+ bias) blocks per matrix
        fragA = 16 * d / 2; sbA = 16 * G * 2 * nsb;
        gateup = 2 * fragA + 2 * sbA;
        slice = d * 8;
        unit = gateup + slice;
        dsc = d * 2;
        dgroup = nsb * dsc;
        expert = uint64_t(dff / 16) * unit + uint64_t(Gd) * dgroup;
    }
    __host__ __device__ uint64_t unit_off(uint32_t u) const { return uint64_t(u) * unit; }
    __host__ __device__ uint64_t group_off(uint32_t gq) const { return uint64_t(dff / 16) * unit + uint64_t(gq) * dgroup; }
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

// grid (d_ff/16 + d_ff/64, n_experts), 256 threads
__global__ void k_prepack(PrepackArgs a) {
    const TiledGeom& t = a.tg;
    const uint32_t e = blockIdx.y, blk = blockIdx.x;
    const uint8_t* s = a.src + uint64_t(e) * a.src_stride;
    uint8_t* dexp = a.dst + uint64_t(e) * a.dst_stride;
    auto NIB = [&](int m) { return s + a.off[3 * m]; };
    auto SC = [&](int m) { return reinterpret_cast<const uint16_t*>(s + a.off[3 * m + 1]); };
    auto BI = [&](int m) { return reinterpret_cast<const uint16_t*>(s + a.off[3 * m + 2]); };
    const bool aff = a.fmt == 1;
    if (blk < t.dff / 16) {
        const uint32_t u = blk, row0 = u * 16;
        uint8_t* p = dexp + t.unit_off(u);
        for (int m = 0; m < 2; ++m) {                       // gate / up fragments
            const uint8_t* nib = NIB(m);
            uint4* frag = reinterpret_cast<uint4*>(p + m * t.fragA);
            for (uint32_t i = threadIdx.x; i < t.G * 32; i += blockDim.x) {
                const uint32_t grp = i >> 5, lane = i & 31, g = lane >> 2, c = lane & 3;
                const uint32_t* rg = reinterpret_cast<const uint32_t*>(nib + size_t(row0 + g) * (t.d / 2) + grp * 32);
                const uint32_t* rh = reinterpret_cast<const uint32_t*>(nib + size_t(row0 + g + 8) * (t.d / 2) + grp * 32);
                frag[i] = make_uint4(rg[c], rh[c], rg[c + 4], rh[c + 4]);
            }
            uint8_t* sb = p + 2 * t.fragA + m * t.sbA;
            for (uint32_t i = threadIdx.x; i < t.G * 16; i += blockDim.x) {
                const uint32_t grp = i >> 4, r = i & 15;
                const uint16_t sc = SC(m)[size_t(row0 + r) * t.G + grp];
                if (aff) reinterpret_cast<uint32_t*>(sb)[i] = sc | (uint32_t(BI(m)[size_t(row0 + r) * t.G + grp]) << 16);
                else reinterpret_cast<uint16_t*>(sb)[i] = sc;
            }
        }
        // down slice: columns 16u..16u+15 of W_down [d x dff]
        uint32_t* sl = reinterpret_cast<uint32_t*>(p + t.gateup);
        const uint8_t* dn = NIB(2);
        for (uint32_t i = threadIdx.x; i < (t.d / 16) * 32; i += blockDim.x) {
            const uint32_t o = i >> 5, L = i & 31, g = L >> 2, c = L & 3;
            const uint8_t* rg = dn + size_t(o * 16 + g) * (t.dff / 2);
            const uint8_t* rh = dn + size_t(o * 16 + g + 8) * (t.dff / 2);
            const uint32_t k0 = row0 + 2 * c, k8 = row0 + 2 * c + 8;
            uint32_t w = 0;
            w |= nib_at(rg, k0) << 0;       w |= nib_at(rg, k0 + 1) << 16;
            w |= nib_at(rh, k0) << 4;       w |= nib_at(rh, k0 + 1) << 20;
            w |= nib_at(rg, k8) << 8;       w |= nib_at(rg, k8 + 1) << 24;
            w |= nib_at(rh, k8) << 12;      w |= nib_at(rh, k8 + 1) << 28;
            sl[i] = w;
        }
    } else {
        const uint32_t gq = blk - t.dff / 16;                  // down scales/biases of group gq
        uint16_t* sc = reinterpret_cast<uint16_t*>(dexp + t.group_off(gq));
        uint16_t* bi = sc + t.d;
        for (uint32_t r = threadIdx.x; r < t.d; r += blockDim.x) {
            sc[r] = SC(2)[size_t(r) * t.Gd + gq];
            if (aff) bi[r] = BI(2)[size_t(r) * t.Gd + gq];
        }
    }
}

}  // namespace smoe
