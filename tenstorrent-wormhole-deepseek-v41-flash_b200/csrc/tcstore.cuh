// Geometry of the tensor-core store ("TC" layout), read by the tcgen05 decode kernel (moe_tc.cu).
//
// Each expert's slice (this GPU's tensor-parallel rows) is cut into the MMA's own tiles, and every
// (tile, 128-K block) -- one pipeline stage of the kernel -- is one contiguous block of bytes, so a
// CTA streams consecutive memory and every stage is a single contiguous read:
//   w1|w3: tile p = 64 rows of w1 then the same 64 rows of w3 (one 128-row MMA tile);
//   w2:    tile m = 128 output rows;
//   block (tile t, K block j) = 128 rows x 128 K in the checkpoint's own byte format, row-major
//     (FP8: 128 bytes per row, e4m3 as stored; FP4: 64 bytes per row, e2m1 packed two per byte, low
//     nibble first), rows or K outside the slice zero. FP4 blocks carry their e8m0 scales inline,
//     512 bytes after the 8192 data bytes, in the order the block-scaled MMA reads them from
//     tensor memory: byte 16 l + 4 c + g is the scale of tile row l + 32 c for K group g (zero
//     outside the slice).
// The TMA tensor engine loads a block with one 128 x 128 box and swizzles it (128-byte swizzle) into
// the canonical K-major layout of tcgen05.mma; FP4 blocks are widened on the way (16U4_ALIGN16B) to
// the padded e2m1 form that kind::mxf8f6f4 reads. FP8 scales live in per-tile tables after the
// blocks, 4 fp32 per (tile, K block):
//   w1|w3: {w1 scale of the 128-row block holding the tile's first row, w1 scale of the next row
//     block, the same two for w3} (a 64-row tile of a slice that starts inside a 128-row block,
//     e.g. 288 rows per GPU at I = 2304, straddles two row blocks);
//   w2: {scale of the global K block holding local K 128 j, scale of the next global K block, 0, 0}
//     (the local K range starts at row0, which need not be a multiple of 128).
#pragma once
#include "common.cuh"

namespace dsmoe {

struct TcGeom {
  int fmt, H, I, row0, I_loc;
  int P1;          // 64-row tiles of w1 (and of w3): ceil(I_loc / 64)
  int KB1;         // 128-K blocks of w1|w3: H / 128
  int KB2;         // 128-K blocks of the w2 slice: ceil(I_loc / 128)
  int MT2;         // 128-row output tiles of w2: H / 128
  int row_bytes;   // bytes of one block row: 128 (FP8) or 64 (FP4)
  long long blk;   // bytes per block: 16384 (FP8) or 8192 + 512 scales (FP4)
  long long d13, s13, eb13;  // w1|w3 blocks, FP8 scale table, expert stride (1 KB multiple)
  long long d2, s2, eb2;     // w2 blocks, FP8 scale table, expert stride
};

__host__ __device__ inline long long tc_round1k(long long v) { return (v + 1023) & ~1023LL; }

__host__ __device__ inline TcGeom tc_geom(int fmt, int H, int I, int row0, int I_loc) {
  TcGeom g;
  g.fmt = fmt;
  g.H = H;
  g.I = I;
  g.row0 = row0;
  g.I_loc = I_loc;
  g.P1 = (I_loc + 63) / 64;
  g.KB1 = H / 128;
  g.KB2 = (I_loc + 127) / 128;
  g.MT2 = H / 128;
  const bool f8 = fmt == DSMOE_FMT_FP8;
  g.row_bytes = f8 ? 128 : 64;
  g.blk = f8 ? 16384 : 8192 + 512;
  g.d13 = (long long)g.P1 * g.KB1 * g.blk;
  g.s13 = f8 ? (long long)g.P1 * g.KB1 * 16 : 0;
  g.eb13 = tc_round1k(g.d13 + g.s13);
  g.d2 = (long long)g.MT2 * g.KB2 * g.blk;
  g.s2 = f8 ? (long long)g.MT2 * g.KB2 * 16 : 0;
  g.eb2 = tc_round1k(g.d2 + g.s2);
  return g;
}

// Shape rules of the TC layout: whole 128-K blocks of hidden, 32-row slice granularity (FP8 w2
// scale segments and FP4 scale groups then split on 32-K steps), an FP4 K a multiple of 32.
__host__ inline bool tc_geom_ok(int fmt, int H, int I, int row0, int I_loc) {
  return (fmt == DSMOE_FMT_FP8 || fmt == DSMOE_FMT_FP4) && H > 0 && H % 128 == 0 && I_loc > 0 && I_loc % 32 == 0 &&
         row0 >= 0 && row0 % 32 == 0 && row0 + I_loc <= I && I % 32 == 0;
}

}  // namespace dsmoe
