// HBM layouts of the grouped FP8 expert path (shared by host and device code).
//
// Swizzled K-major tile (the tensor cores' shared-memory image, SWIZZLE_128B): 128 rows x 128
// bytes of K, row r at byte 128 r, its 16-byte chunk c stored at chunk position c ^ (r & 7).
// Eight rows (1024 B) form one swizzle atom; a TMA bulk copy of a tile into a 1024-byte
// aligned stage gives exactly the operand a tcgen05 smem descriptor describes.
//
// Expert arena (one slot per resident expert, written once at upload by relayout.cu):
//   [ up/gate tiles | down tiles | scale grids ]
//   up/gate: for 128-row block rb (of I) and 128-column block kb (of H), 32 KB =
//     [w_up tile | w_gate tile], tiles of one rb contiguous over kb -> the work item
//     (group, rb) streams rb's row of tiles front to back.
//   down: the same with one 16 KB w_down tile per (rb of H, kb of I).
//   scale grids: w_up, w_gate [I/128, H/128] and w_down [H/128, I/128] fp32, row-major
//     exactly as in the upload format (expert_format_v2.h BlockScaleMetaV2).
//
// Packed activations (per layer call, written by pack_act.cu):
//   rows are grouped; a group is <= 16 rows of one expert slot (NT = 1 or 2 n-tiles of 8).
//   For group g and K block kb the B operand is one swizzled K-major tile of 3 * 8 NT rows
//   (row n = term * 8 NT + token, term = 0..2 of the three-term E4M3 split) at byte
//       (tile_base(g) * KB + kb * NT) * 3072,
//   and the power-of-two scale of (token, kb) is the float at
//       (tile_base(g) * KB + kb * NT) * 8 + token.
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
    int32_t split_k;   // K split the up/gate kernel chose (read by the h packer)
    int32_t pad[3];
};

}  // namespace cst
