// HBM layouts of the grouped FP8 expert path (shared by host and device code).
//
// Expert arena (one slot per resident expert, written once at upload):
//   [ up/gate chunks | down chunks | scale grids ]
//   up/gate chunk (mb, kb): the 64 rows [64 mb, 64 mb + 64) of BOTH w_up and w_gate over
//     the 128 columns of K block kb, 16 KB, fragment-major:
//       byte = ((w * 4 + ks) * 2 + mat) * 512 + lane * 16 + j
//     w = consumer warp (16 rows each), ks = 32-wide k step, mat = 0 up / 1 gate,
//     lane = 4 g + t, j = 4 reg + byte with reg 0..3 the mma.m16n8k32 A registers:
//       row = 16 w + g + 8 (reg & 1),  col = 32 ks + 4 t + 16 (reg >> 1) + byte.
//     Chunks of one 64-row item are contiguous: one TMA bulk copy per K block.
//   down chunk (mb, kb): the same with one matrix (w_down rows = hidden), 8 KB.
//   scale grids: w_up, w_gate [I/128, H/128] and w_down [H/128, I/128] fp32, row-major
//     exactly as in the upload format (expert_format_v2.h BlockScaleMetaV2).
//
// Packed activations (per layer call, written by the activation packer):
//   rows are grouped; a group is <= 16 rows of one expert slot (2 n-tiles of 8);
//   for n-tile `tile` (global tile index) and K block kb the B operand is
//       ((tile_base_of_group * KB + kb * NT + nt) * 3072) + (ks * 3 + split) * 256 + lane * 8 + j
//     lane = 4 g + t, j = 4 half + byte:  token col = g, k = 32 ks + 4 t + 16 half + byte
//   and the per-(row, K block) power-of-two scale sits at
//       (tile_base_of_group * KB + kb * NT + nt) * 8 + col.
#pragma once

#include <cstddef>
#include <cstdint>

namespace cst {

struct ArenaGeom {
    int hidden;   // H
    int inter;    // I
    int64_t upgate_bytes;
    int64_t down_bytes;
    int64_t su_off, sg_off, sd_off;  // byte offsets of the scale grids inside a slot
    int64_t slot_bytes;

    static inline int64_t align_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

    static ArenaGeom make(int hidden, int inter) {
        ArenaGeom g{};
        g.hidden = hidden;
        g.inter = inter;
        g.upgate_bytes = int64_t(2) * inter * hidden;
        g.down_bytes = int64_t(inter) * hidden;
        const int64_t ngrid = int64_t(inter / 128) * (hidden / 128);
        g.su_off = g.upgate_bytes + g.down_bytes;
        g.sg_off = g.su_off + align_up(ngrid * 4, 256);
        g.sd_off = g.sg_off + align_up(ngrid * 4, 256);
        g.slot_bytes = align_up(g.sd_off + align_up(ngrid * 4, 256), 4096);
        return g;
    }
};

// Per-group record produced by the router packer.
struct GroupRec {
    int32_t slot;       // expert slot in the arena
    int32_t row_start;  // first packed row
    int32_t n_rows;     // 1..16
    int32_t tile_base;  // first global n-tile index
};

// Meta block written by the packer (device) and read back by the host when needed.
struct PackMeta {
    int32_t n_rows;
    int32_t n_groups;
    int32_t n_tiles;
    int32_t overflow;  // nonzero: the call exceeded the workspace capacity
};

}  // namespace cst
