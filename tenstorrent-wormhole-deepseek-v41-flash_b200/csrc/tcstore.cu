// Pack / unpack of the tensor-core store (layout in tcstore.cuh): one expert's slice of checkpoint
// tensors (device memory) -> its w1|w3 part and its w2 part, cut into contiguous (tile, K block)
// blocks of the checkpoint's own bytes, with the FP8 scales in per-tile tables and the FP4 scales
// inline after each block. The reference kept experts in host files of Tenstorrent tiles packed on
// demand (dsv41/tt/store.py:66-120, dsv41/ref/fp4lib.c:116-186); here the layout is the decode
// kernel's pipeline stage, so each stage is one contiguous read.
#include "tcstore.cuh"

namespace dsmoe {

// Block data, 16 bytes per thread. MODE 13: w1|w3 blocks (rows 0..63 of a tile from w1, 64..127
// from w3); MODE 2: w2 blocks (128 output rows; K = the slice's columns, from row0).
template <int MODE>
__global__ void tc_pack_blocks(TcGeom g, const uint8_t* sa, const uint8_t* sb, uint8_t* dst) {
  const int cpr = g.row_bytes / 16;                 // 16-byte chunks per block row
  const long long cpb = 128LL * cpr;                // per block
  const int KB = MODE == 13 ? g.KB1 : g.KB2;
  const long long n = (long long)(MODE == 13 ? g.P1 : g.MT2) * KB * cpb;
  const bool f8 = g.fmt == DSMOE_FMT_FP8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long b = i / cpb;
    const int c = (int)(i - b * cpb), R = c / cpr, cc = c - R * cpr;
    const int t = (int)(b / KB), j = (int)(b - (long long)t * KB);
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (MODE == 13) {
      const int r = 64 * t + (R & 63);
      if (r < g.I_loc) {
        const uint8_t* s = R < 64 ? sa : sb;
        const long long k13 = f8 ? g.H : g.H / 2;
        v = *reinterpret_cast<const uint4*>(s + (long long)(g.row0 + r) * k13 + (long long)j * g.row_bytes + 16 * cc);
      }
    } else {
      const int kel = 128 * j + (f8 ? 16 : 32) * cc;  // first local K element of the chunk
      if (kel < g.I_loc) {
        const long long pitch = f8 ? g.I : g.I / 2, col0 = f8 ? g.row0 : g.row0 / 2;
        v = *reinterpret_cast<const uint4*>(sa + (long long)(128 * t + R) * pitch + col0 + (long long)j * g.row_bytes +
                                            16 * cc);
      }
    }
    *reinterpret_cast<uint4*>(dst + b * g.blk + (long long)R * g.row_bytes + 16 * cc) = v;
  }
}

// FP8 w1|w3 scale table: [P1][KB1][4] fp32 (see tcstore.cuh).
__global__ void tc_pack_s13_fp8(TcGeom g, const float* s1, const float* s3, float* dst) {
  const int n = g.P1 * g.KB1;
  const int rb = (g.I + 127) / 128;  // row blocks of the full expert
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int p = i / g.KB1, kb = i - p * g.KB1;
    const int first = g.row0 + 64 * p, last = g.row0 + min(64 * p + 63, g.I_loc - 1);
    const int b0 = first >> 7, b1 = min(last >> 7, rb - 1);
    float4 v;
    v.x = s1[(long long)b0 * g.KB1 + kb];
    v.y = s1[(long long)b1 * g.KB1 + kb];
    v.z = s3[(long long)b0 * g.KB1 + kb];
    v.w = s3[(long long)b1 * g.KB1 + kb];
    reinterpret_cast<float4*>(dst)[i] = v;
  }
}

// FP8 w2 scale table: [MT2][KB2][4] fp32.
__global__ void tc_pack_s2_fp8(TcGeom g, const float* s2, float* dst) {
  const int n = g.MT2 * g.KB2;
  const int kbg = (g.I + 127) / 128;  // K blocks of the full expert
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int m = i / g.KB2, kb = i - m * g.KB2;
    const int g0 = (g.row0 + 128 * kb) >> 7, g1 = min(g0 + 1, kbg - 1);
    reinterpret_cast<float4*>(dst)[i] = make_float4(s2[(long long)m * kbg + g0], s2[(long long)m * kbg + g1], 0.f, 0.f);
  }
}

// FP4 scales inline after each block's data: byte 16 l + 4 c + gq = scale of tile row l + 32 c, K
// group 4 kb + gq. MODE 13: tile = 64-row pair tile (rows 0..63 w1, 64..127 w3), source [I][H/32];
// MODE 2: tile = 128 output rows of w2, source [H][I/32] (K groups offset by row0 / 32).
template <int MODE>
__global__ void tc_pack_sf_fp4(TcGeom g, const uint8_t* sa, const uint8_t* sb, uint8_t* dst) {
  const int tiles = MODE == 13 ? g.P1 : g.MT2, KB = MODE == 13 ? g.KB1 : g.KB2;
  const long long n = (long long)tiles * KB * 512;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int byte = (int)(i & 511);
    const long long tk = i >> 9;
    const int t = (int)(tk / KB), kb = (int)(tk - (long long)t * KB);
    const int l = byte >> 4, c = (byte >> 2) & 3, gq = byte & 3;
    const int R = l + 32 * c;
    uint8_t v = 0;
    if (MODE == 13) {
      const int r = 64 * t + (R & 63);
      if (r < g.I_loc) {
        const uint8_t* s = R < 64 ? sa : sb;
        v = s[(long long)(g.row0 + r) * (g.H / 32) + 4 * kb + gq];
      }
    } else {
      const int q = 4 * kb + gq;  // local K group
      if (32 * q < g.I_loc) v = sa[(long long)(128 * t + R) * (g.I / 32) + g.row0 / 32 + q];
    }
    dst[tk * g.blk + 8192 + byte] = v;
  }
}

// Dequantize a packed expert back to fp32 slices (w1, w3 [I_loc, H], w2 [H, I_loc]) through the
// scale tables, the way the decode kernel reads them: proves the layout lossless.
__global__ void tc_unpack_kernel(TcGeom g, const uint8_t* w13, const uint8_t* w2b, float* w1, float* w3, float* w2) {
  const long long n13 = 2LL * g.I_loc * g.H, n2 = (long long)g.H * g.I_loc;
  const bool f8 = g.fmt == DSMOE_FMT_FP8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n13 + n2; i += (long long)gridDim.x * blockDim.x) {
    float v;
    if (i < n13) {
      const int m = (int)(i / ((long long)g.I_loc * g.H));
      const long long rk = i - (long long)m * g.I_loc * g.H;
      const int r = (int)(rk / g.H), k = (int)(rk - (long long)r * g.H);
      const int p = r >> 6, kb = k >> 7, R = (r & 63) + 64 * m, kk = k & 127;
      const uint8_t* blk = w13 + ((long long)p * g.KB1 + kb) * g.blk;
      if (f8) {
        const uint8_t b = blk[R * 128 + kk];
        const float* st = reinterpret_cast<const float*>(w13 + g.d13) + ((long long)p * g.KB1 + kb) * 4;
        const bool second = ((g.row0 + r) >> 7) != ((g.row0 + 64 * p) >> 7);
        v = f16_lo(e4m3x2_to_f16x2(b)) * st[2 * m + (second ? 1 : 0)];
      } else {
        const uint8_t b = blk[R * 64 + (kk >> 1)];
        const uint8_t sf = blk[8192 + 16 * (R & 31) + 4 * (R >> 5) + (kk >> 5)];
        const uint32_t h2 = e2m1x2_to_f16x2(b);
        v = ((k & 1) ? f16_hi(h2) : f16_lo(h2)) * e8m0_to_f32(sf);
      }
      (m == 0 ? w1 : w3)[(long long)r * g.H + k] = v;
    } else {
      const long long j = i - n13;
      const int nrow = (int)(j / g.I_loc), k = (int)(j - (long long)nrow * g.I_loc);
      const int mt = nrow >> 7, kb = k >> 7, R = nrow & 127, kk = k & 127;
      const uint8_t* blk = w2b + ((long long)mt * g.KB2 + kb) * g.blk;
      if (f8) {
        const uint8_t b = blk[R * 128 + kk];
        const float* st = reinterpret_cast<const float*>(w2b + g.d2) + ((long long)mt * g.KB2 + kb) * 4;
        const bool second = ((g.row0 + k) >> 7) != ((g.row0 + 128 * kb) >> 7);
        v = f16_lo(e4m3x2_to_f16x2(b)) * st[second ? 1 : 0];
      } else {
        const uint8_t b = blk[R * 64 + (kk >> 1)];
        const uint8_t sf = blk[8192 + 16 * (R & 31) + 4 * (R >> 5) + (kk >> 5)];
        const uint32_t h2 = e2m1x2_to_f16x2(b);
        v = ((k & 1) ? f16_hi(h2) : f16_lo(h2)) * e8m0_to_f32(sf);
      }
      w2[(long long)nrow * g.I_loc + k] = v;
    }
  }
}

}  // namespace dsmoe

using namespace dsmoe;

extern "C" int dsmoe_store_tc_expert_bytes(int fmt, int hidden, int inter, int row0, int inter_local,
                                           long long* w13_bytes, long long* w2_bytes) {
  DSMOE_REQUIRE(w13_bytes && w2_bytes, DSMOE_ERR_ARG, "store_tc_expert_bytes: null pointer");
  DSMOE_REQUIRE(tc_geom_ok(fmt, hidden, inter, row0, inter_local), DSMOE_ERR_ARG,
                "store_tc: fmt %d, hidden %d (multiple of 128), slice [%d, %d) of %d (multiples of 32)", fmt, hidden,
                row0, row0 + inter_local, inter);
  const TcGeom g = tc_geom(fmt, hidden, inter, row0, inter_local);
  *w13_bytes = g.eb13;
  *w2_bytes = g.eb2;
  return DSMOE_OK;
}

extern "C" int dsmoe_store_tc_pack_expert(int fmt, int hidden, int inter, int row0, int inter_local,
                                          const uint8_t* w1, const void* s1, const uint8_t* w3, const void* s3,
                                          const uint8_t* w2, const void* s2, uint8_t* w13_dst, uint8_t* w2_dst,
                                          void* stream) {
  DSMOE_REQUIRE(tc_geom_ok(fmt, hidden, inter, row0, inter_local), DSMOE_ERR_ARG,
                "store_tc_pack: fmt %d, hidden %d, slice [%d, %d) of %d", fmt, hidden, row0, row0 + inter_local, inter);
  DSMOE_REQUIRE(w1 && s1 && w3 && s3 && w2 && s2 && w13_dst && w2_dst, DSMOE_ERR_ARG, "store_tc_pack: null pointer");
  DSMOE_REQUIRE((((uintptr_t)w13_dst | (uintptr_t)w2_dst) & 1023) == 0, DSMOE_ERR_ALIGN,
                "store_tc_pack: destinations must be 1024-byte aligned");
  DSMOE_REQUIRE((((uintptr_t)w1 | (uintptr_t)w3 | (uintptr_t)w2) & 15) == 0, DSMOE_ERR_ALIGN,
                "store_tc_pack: weight sources must be 16-byte aligned");
  const TcGeom g = tc_geom(fmt, hidden, inter, row0, inter_local);
  cudaStream_t st = (cudaStream_t)stream;
  const int T = 256;
  auto grid = [&](long long n) { return (int)std::min<long long>((n + T - 1) / T, 148 * 16); };
  tc_pack_blocks<13><<<grid((long long)g.P1 * g.KB1 * 128 * (g.row_bytes / 16)), T, 0, st>>>(g, w1, w3, w13_dst);
  tc_pack_blocks<2><<<grid((long long)g.MT2 * g.KB2 * 128 * (g.row_bytes / 16)), T, 0, st>>>(g, w2, nullptr, w2_dst);
  if (fmt == DSMOE_FMT_FP8) {
    tc_pack_s13_fp8<<<(g.P1 * g.KB1 + T - 1) / T, T, 0, st>>>(g, (const float*)s1, (const float*)s3,
                                                              (float*)(w13_dst + g.d13));
    tc_pack_s2_fp8<<<(g.MT2 * g.KB2 + T - 1) / T, T, 0, st>>>(g, (const float*)s2, (float*)(w2_dst + g.d2));
  } else {
    tc_pack_sf_fp4<13><<<grid((long long)g.P1 * g.KB1 * 512), T, 0, st>>>(g, (const uint8_t*)s1, (const uint8_t*)s3,
                                                                          w13_dst);
    tc_pack_sf_fp4<2><<<grid((long long)g.MT2 * g.KB2 * 512), T, 0, st>>>(g, (const uint8_t*)s2, nullptr, w2_dst);
  }
  return cuda_status("store_tc_pack");
}

extern "C" int dsmoe_store_tc_unpack_expert(int fmt, int hidden, int inter, int row0, int inter_local,
                                            const uint8_t* w13_src, const uint8_t* w2_src, float* w1, float* w3,
                                            float* w2, void* stream) {
  DSMOE_REQUIRE(tc_geom_ok(fmt, hidden, inter, row0, inter_local), DSMOE_ERR_ARG, "store_tc_unpack: bad geometry");
  DSMOE_REQUIRE(w13_src && w2_src && w1 && w3 && w2, DSMOE_ERR_ARG, "store_tc_unpack: null pointer");
  const TcGeom g = tc_geom(fmt, hidden, inter, row0, inter_local);
  tc_unpack_kernel<<<148 * 8, 256, 0, (cudaStream_t)stream>>>(g, w13_src, w2_src, w1, w3, w2);
  return cuda_status("store_tc_unpack");
}
