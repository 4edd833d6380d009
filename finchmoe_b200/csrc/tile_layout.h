// Device-side layout of a routed 3-bit expert block inside the HBM pool.
//
// The pool does not keep the on-disk byte order (finchmoe/infer.m:223-234).
// finch_pool_put() re-tiles a block into *tiles*: the 16 matrix rows one warp
// feeds to the tensor cores as one MMA tile, stored contiguously (one bulk
// copy per tile) and ordered so that every lane reads its operand words from
// consecutive shared-memory addresses (no bank conflicts, no padding):
//
//   tile (16 fragment rows; lane (g, t) owns fragment rows g ("A") and g + 8 ("B"))
//     weights [units][32 lanes][6 words]   3 words of row A then 3 words of row B, both for
//                                          period t of unit u (row words 12u + 3t .. + 2)
//     sb      [units][8 g][4 words]        scale word of row A, of row B, bias word of row A,
//                                          of row B (one word = the two groups of unit u)
//   A-tile ta (gate/up): row A = gate row 8*ta + g, row B = up row 8*ta + g   (K = hidden)
//   B-tile tb (down):    row A = down row 16*tb + g, row B = down row 16*tb + 8 + g (K = inter)
//
// block = nTA A-tiles, then nTB B-tiles; the size equals the on-disk block size.
// finch_pool_get() applies the inverse permutation, so callers only ever see
// the reference's byte order.
#pragma once
#include <stddef.h>
#include <stdint.h>

#if defined(__CUDACC__)
#define FINCH_HD __host__ __device__
#else
#define FINCH_HD
#endif

struct FinchTile {
    int unitsA, unitsD, nTA, nTB;
    int tileA, tileB;    // bytes per tile
    int sbA, sbB;        // byte offset of the scale/bias entries inside a tile
    size_t b_base;       // byte offset of the first B-tile
    size_t total;
};

FINCH_HD inline FinchTile finch_tile(int hidden, int inter) {
    FinchTile T;
    T.unitsA = hidden / 128;
    T.unitsD = inter / 128;
    T.nTA = inter / 8;
    T.nTB = hidden / 16;
    T.sbA = T.unitsA * 768;
    T.sbB = T.unitsD * 768;
    T.tileA = T.unitsA * 896;
    T.tileB = T.unitsD * 896;
    T.b_base = (size_t)T.nTA * T.tileA;
    T.total = T.b_base + (size_t)T.nTB * T.tileB;
    return T;
}

// Reference (on-disk) offsets of the nine regions.
struct FinchDisk {
    size_t gate_w, gate_s, gate_b, up_w, up_s, up_b, down_w, down_s, down_b, size;
};
FINCH_HD inline FinchDisk finch_disk(int hidden, int inter) {
    FinchDisk D;
    const size_t gw = (size_t)inter * hidden * 3 / 8, gs = (size_t)inter * (hidden / 64) * 2;
    const size_t ds = (size_t)hidden * (inter / 64) * 2;
    D.gate_w = 0;
    D.gate_s = gw;
    D.gate_b = gw + gs;
    D.up_w = gw + 2 * gs;
    D.up_s = D.up_w + gw;
    D.up_b = D.up_s + gs;
    D.down_w = D.up_b + gs;
    D.down_s = D.down_w + gw;
    D.down_b = D.down_s + ds;
    D.size = D.down_b + ds;
    return D;
}

// Host only.  One call moves every 32-bit word between the two layouts.
// to_device != 0: disk -> tiled; else tiled -> disk.
inline void finch_retile(int hidden, int inter, const uint8_t *src, uint8_t *dst, int to_device) {
    const FinchTile T = finch_tile(hidden, inter);
    const FinchDisk D = finch_disk(hidden, inter);
    const uint32_t *s32 = (const uint32_t *)src;
    uint32_t *d32 = (uint32_t *)dst;
    auto mv = [&](size_t disk_byte, size_t tile_byte) {
        if (to_device) d32[tile_byte / 4] = s32[disk_byte / 4];
        else d32[disk_byte / 4] = s32[tile_byte / 4];
    };
    const size_t rowA = (size_t)hidden * 3 / 8, rowD = (size_t)inter * 3 / 8;
    const size_t sA = (size_t)(hidden / 64) * 2, sD = (size_t)(inter / 64) * 2;
    for (int ta = 0; ta < T.nTA; ta++) {
        const size_t tb = (size_t)ta * T.tileA;
        for (int g = 0; g < 8; g++) {
            const size_t r = (size_t)8 * ta + g;
            for (int u = 0; u < T.unitsA; u++) {
                for (int t = 0; t < 4; t++)
                    for (int k = 0; k < 3; k++) {
                        const size_t lane_off = tb + (((size_t)u * 32 + g * 4 + t) * 6) * 4;
                        mv(D.gate_w + r * rowA + (12 * u + 3 * t + k) * 4, lane_off + k * 4);
                        mv(D.up_w + r * rowA + (12 * u + 3 * t + k) * 4, lane_off + (3 + k) * 4);
                    }
                const size_t e = tb + T.sbA + (((size_t)u * 8 + g) * 4) * 4;
                mv(D.gate_s + r * sA + u * 4, e);
                mv(D.up_s + r * sA + u * 4, e + 4);
                mv(D.gate_b + r * sA + u * 4, e + 8);
                mv(D.up_b + r * sA + u * 4, e + 12);
            }
        }
    }
    for (int t2 = 0; t2 < T.nTB; t2++) {
        const size_t tb = T.b_base + (size_t)t2 * T.tileB;
        for (int g = 0; g < 8; g++) {
            const size_t r0 = (size_t)16 * t2 + g, r1 = r0 + 8;
            for (int u = 0; u < T.unitsD; u++) {
                for (int t = 0; t < 4; t++)
                    for (int k = 0; k < 3; k++) {
                        const size_t lane_off = tb + (((size_t)u * 32 + g * 4 + t) * 6) * 4;
                        mv(D.down_w + r0 * rowD + (12 * u + 3 * t + k) * 4, lane_off + k * 4);
                        mv(D.down_w + r1 * rowD + (12 * u + 3 * t + k) * 4, lane_off + (3 + k) * 4);
                    }
                const size_t e = tb + T.sbB + (((size_t)u * 8 + g) * 4) * 4;
                mv(D.down_s + r0 * sD + u * 4, e);
                mv(D.down_s + r1 * sD + u * 4, e + 4);
                mv(D.down_b + r0 * sD + u * 4, e + 8);
                mv(D.down_b + r1 * sD + u * 4, e + 12);
            }
        }
    }
}

// ---- shared expert (4-bit affine), prepared copy --------------------------
// The caller hands the shared expert over in the reference's tensor layout
// (finchmoe/quantize_non_experts.py:57-65).  Before first use it is re-tiled
// on the device into tiles of the same kind:
//   gate/up tile (4 gate rows + the 4 matching up rows; lanes g and g + 4 read the same data)
//     weights [groups][16 (g&3, t)][4 words]   words 2t, 2t+1 of the gate row, then of the up row
//     sb      [groups][4][4 x u16]             scale gate, scale up, bias gate, bias up
//   down tile (16 rows; lane rows g and g + 8)
//     weights [groups][32][4 words], sb [groups][8][4 x u16]
struct FinchTile4 {
    int groupsA, groupsD, nTA, nTB;
    int tileA, tileB, sbA, sbB;
    size_t b_base, total;
};
FINCH_HD inline FinchTile4 finch_tile4(int hidden, int inter) {
    FinchTile4 T;
    T.groupsA = hidden / 64;
    T.groupsD = inter / 64;
    T.nTA = inter / 4;
    T.nTB = hidden / 16;
    T.sbA = T.groupsA * 256;
    T.tileA = T.groupsA * (256 + 32);
    T.sbB = T.groupsD * 512;
    T.tileB = T.groupsD * (512 + 64);
    T.b_base = (size_t)T.nTA * T.tileA;
    T.total = T.b_base + (size_t)T.nTB * T.tileB;
    return T;
}
