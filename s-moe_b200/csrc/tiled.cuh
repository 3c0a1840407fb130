// tiled.cuh - the tiled expert layout and its one-time prepack kernel.
//
// Vault layout (shatter_moe.py:627-674): per matrix, row-major nibbles then
// row-major scales (then biases for AFFINE-Q4). Reading a 16-row tile of it
// needs one copy per row (1 KB or 384 B), and 1-D bulk copies that small run
// far below the HBM roofline on B200 (measured: 384 B -> 1.9 TB/s, >= 2 KB ->
// 5.5 TB/s over 148 SMs). The tiled layout makes every unit of work of the
// fused kernel one contiguous block:
//   expert = [A tile 0 .. A tile d_ff/16-1][B tile 0 .. B tile d_model/16-1]
//   A tile = [gate frag][up frag][gate sc^T][up sc^T][gate bias^T][up bias^T]
//   B tile = [down frag][down sc^T][down bias^T]
// frag: the 16 x cols nibble tile in MMA-fragment order - for each 64-group,
//   256 B for rows 0-7 then 256 B for rows 8-15, lane L's 8 bytes at L*8
//   (row L/4, bytes 8*(L%4)..+7 of the group) - so a warp's fragment loads
//   are consecutive in shared memory (no bank conflicts, no padding).
// sc^T / bias^T: the tile's per-group values transposed to [group][16 rows].
// Biases exist for AFFINE-Q4 only. Byte count equals the vault layout's.
#pragma once
#include "smoe_common.cuh"

namespace smoe {

struct TiledGeom {
    uint32_t d, dff, G, Gd;
    uint32_t fragA, scA, tileA;     // bytes: one matrix frag, one sc^T block, whole A tile
    uint32_t fragB, scB, tileB;
    uint64_t expert;
    __host__ __device__ void init(int fmt, uint32_t d_, uint32_t dff_) {
        d = d_; dff = dff_; G = d / 64; Gd = dff / 64;
        const uint32_t nsb = (fmt == 1) ? 2 : 1;            // scale (+ bias) blocks per matrix
        fragA = 16 * d / 2; scA = 16 * G * 2;
        tileA = 2 * fragA + 2 * nsb * scA;
        fragB = 16 * dff / 2; scB = 16 * Gd * 2;
        tileB = fragB + nsb * scB;
        expert = uint64_t(dff / 16) * tileA + uint64_t(d / 16) * tileB;
    }
    __host__ __device__ uint64_t a_tile(uint32_t t) const { return uint64_t(t) * tileA; }
    __host__ __device__ uint64_t b_tile(uint32_t t) const { return uint64_t(dff / 16) * tileA + uint64_t(t) * tileB; }
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

// One 16-row tile of one matrix: fragments + transposed scales/biases.
SMOE_DEVINL void pack_tile(const uint8_t* nib, const uint16_t* sc, const uint16_t* bi, uint32_t cols,
                           uint32_t row0, uint8_t* frag, uint16_t* scT, uint16_t* biT) {
    const uint32_t G = cols / 64;
    for (uint32_t i = threadIdx.x; i < G * 64; i += blockDim.x) {      // uint2 units
        const uint32_t grp = i >> 6, half = (i >> 5) & 1, lane = i & 31;
        const uint32_t row = row0 + half * 8 + (lane >> 2);
        const uint2 v = *reinterpret_cast<const uint2*>(nib + size_t(row) * (cols / 2) + grp * 32 + (lane & 3) * 8);
        reinterpret_cast<uint2*>(frag)[i] = v;
    }
    for (uint32_t i = threadIdx.x; i < G * 16; i += blockDim.x) {
        const uint32_t grp = i >> 4, r = i & 15;
        scT[i] = sc[size_t(row0 + r) * G + grp];
        if (biT) biT[i] = bi[size_t(row0 + r) * G + grp];
    }
}

// grid (d_ff/16 + d_model/16, n_experts), 256 threads
__global__ void k_prepack(PrepackArgs a) {
    const TiledGeom& t = a.tg;
    const uint32_t e = blockIdx.y, tile = blockIdx.x;
    const uint8_t* s = a.src + uint64_t(e) * a.src_stride;
    uint8_t* dexp = a.dst + uint64_t(e) * a.dst_stride;
    auto NIB = [&](int m) { return s + a.off[3 * m]; };
    auto SC = [&](int m) { return reinterpret_cast<const uint16_t*>(s + a.off[3 * m + 1]); };
    auto BI = [&](int m) { return reinterpret_cast<const uint16_t*>(s + a.off[3 * m + 2]); };
    const bool aff = a.fmt == 1;
    if (tile < t.dff / 16) {
        uint8_t* p = dexp + t.a_tile(tile);
        for (int m = 0; m < 2; ++m) {
            uint16_t* scT = reinterpret_cast<uint16_t*>(p + 2 * t.fragA + m * t.scA);
            uint16_t* biT = aff ? reinterpret_cast<uint16_t*>(p + 2 * t.fragA + (2 + m) * t.scA) : nullptr;
            pack_tile(NIB(m), SC(m), BI(m), t.d, tile * 16, p + m * t.fragA, scT, biT);
        }
    } else {
        const uint32_t bt = tile - t.dff / 16;
        uint8_t* p = dexp + t.b_tile(bt);
        uint16_t* scT = reinterpret_cast<uint16_t*>(p + t.fragB);
        uint16_t* biT = aff ? reinterpret_cast<uint16_t*>(p + t.fragB + t.scB) : nullptr;
        pack_tile(NIB(2), SC(2), BI(2), t.dff, bt * 16, p, scT, biT);
    }
}

}  // namespace smoe
