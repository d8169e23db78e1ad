// Tile records: the device layout of a packed int4 matrix for the B200 kernels.
//
// The reference stores a stacked linear as packed [E][R][K/8] int32 (column
// i + 8m = nibble i of word m), scale [E][R][G] and, here, optional zero points
// [E][R][ceil(G/8)].  `duplex_repack_tiles` rewrites it once into one record per
// (expert, block of 16 rows); a kernel stage is one record (one bulk copy), and
// every thread reads its MMA fragments with one conflict-free 16-byte load:
//
//   weights  npairs x [32 lanes][4 words]   pair p = columns [64p, 64p + 64)
//            lane (g = lane/4, t = lane%4) holds the words
//              { row g    word 8p+t,   row g+8 word 8p+t,
//                row g    word 8p+4+t, row g+8 word 8p+4+t }
//            i.e. the 32-column windows 2p and 2p+1 of rows g and g+8
//   scales   Gr x [8 g][row g, row g+8]  (16-bit, the stored scale dtype)
//   zeros    Gr x [8 g] bytes: z(row g) | z(row g+8) << 4      (only if zero points)
//   padding  to a multiple of 128 bytes
//
// K is padded to a multiple of 64 with zero nibbles (their activations are zero),
// Gr = ceil(Kp / group) groups (padded groups have scale 0), rows past R are zero.
// With `pair_halves` (gate|up stacks) the records of row block j of the first half
// and row block j of the second half are adjacent, so one copy brings a gate block
// and its up block.
#pragma once

#include <stddef.h>
#include <stdint.h>

namespace duplex {

struct TileGeom {
  int K;          // logical columns
  int Kp;         // padded to 64
  int npairs;     // Kp / 64
  int Gr;         // groups stored per record
  int group;      // 32 or 64 * 2^k
  int gshift;     // pairs per group = 1 << gshift (group >= 64); -1 for group 32
  int has_zeros;
  uint32_t off_scale, off_zero, rec_bytes;
};

inline int tile_geom(int K, int group, int has_zeros, TileGeom* t) {
  if (K < 32 || (K & 31) || group < 32) return 1;
  int gshift;
  if (group == 32) {
    gshift = -1;
  } else {
    if (group % 64) return 1;
    int q = group / 64, s = 0;
    while ((1 << s) < q) ++s;
    if ((1 << s) != q) return 1;
    gshift = s;
  }
  t->K = K;
  t->Kp = (K + 63) / 64 * 64;
  t->npairs = t->Kp / 64;
  t->group = group;
  t->gshift = gshift;
  t->Gr = (t->Kp + group - 1) / group;
  t->has_zeros = has_zeros ? 1 : 0;
  t->off_scale = (uint32_t)t->npairs * 512u;
  t->off_zero = t->off_scale + (uint32_t)t->Gr * 32u;
  const uint32_t end = t->off_zero + (has_zeros ? (uint32_t)t->Gr * 8u : 0u);
  t->rec_bytes = (end + 127u) / 128u * 128u;
  return 0;
}

}  // namespace duplex
