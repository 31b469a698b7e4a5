// Resident expert store: one-time repack of checkpoint-layout experts into the tensor-core
// fragment order the decode kernels stream, scales co-located with their weight tiles.
//
// Replaces the reference's host-side store (dsv41/tt/store.py:66-120: per-(layer, expert, proj)
// files packed on demand, paged into 6 device slots per layer) and its tile packer
// (dsv41/ref/fp4lib.c:116-186). Here every expert of a layer is resident in HBM, repacked once on
// the device, so there is no paging and no per-token gather (the reference's SlotCat gather,
// dsv41/kernels/slot_cat.cpp:194-365, has no counterpart).
//
// Lane chunk layout (lane l: g = l / 4, t = l % 4; rows relative to a 16-row tile), built around
// the A operand of mma.m16n8k32 with 8-bit inputs (four 32-bit registers, 4 consecutive K each:
// a0 = row g, K 4t..4t+3; a1 = row g+8, same K; a2 = row g, K 16+4t..; a3 = row g+8, K 16+4t..):
//  FP8, 32 K per chunk, 16 bytes per lane: byte 4r + i (r = register 0..3, i = 0..3) holds
//      row g + 8*(r & 1), K = 4t + i + 16*(r >> 1)          -- the A fragment itself
//  FP4, 64 K per chunk (two MMAs), 16 bytes per lane = words w = 0..3, byte i of word w holds two
//      codes of row g + 8*(w & 1): low nibble K = 32*(w >> 1) + 4t + i, high nibble that K + 16.
//      A word expands to two A registers of e4m3 (low nibbles -> a0 / a1, high -> a2 / a3) with
//      four integer operations (fp4x8_to_e4m3).
//  FP4 chunk scales, 32 bytes: byte 4g + q: q 0 (g, group 2c), 1 (g, 2c+1), 2 (g+8, 2c), 3 (g+8, 2c+1)
// FP8 chunks are grouped 8 to an item with the item's scales right after (common.cuh).
#include "common.cuh"

namespace dsmoe {

struct PackArgs {
  int fmt, H, I, row0, I_loc;
  const uint8_t *w1, *w3, *w2;
  const void *s1, *s3, *s2;
  uint8_t *w13, *w2d;
};

__device__ __forceinline__ void lane_rows_fp8(int l, int j, int& row, int& k) {
  const int g = l >> 2, t = l & 3, r = j >> 2, i = j & 3;
  row = g + 8 * (r & 1);
  k = 4 * t + i + 16 * (r >> 1);
}
// FP4: the low-nibble code's K; the high nibble holds K + 16 of the same row
__device__ __forceinline__ void lane_rows_fp4(int l, int j, int& row, int& k) {
  const int g = l >> 2, t = l & 3, w = j >> 2, i = j & 3;
  row = g + 8 * (w & 1);
  k = 32 * (w >> 1) + 4 * t + i;
}
// e2m1 code of (row, k) from a checkpoint-layout FP4 row (low nibble = even k)
__device__ __forceinline__ uint32_t fp4_code(const uint8_t* rowp, int k) {
  return (rowp[k >> 1] >> (4 * (k & 1))) & 0xF;
}

// One thread per (tile, chunk, matrix, lane) 16-byte output.
__global__ void pack_w13_kernel(PackArgs a) {
  const int T = a.I_loc / 16;
  const int KC = a.fmt == DSMOE_FMT_FP8 ? a.H / 32 : a.H / 64;
  const long long tile_b = w13_tile_bytes(a.fmt, a.H);
  const long long total = (long long)T * KC * 2 * 32;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int l = i & 31, m = (i >> 5) & 1;
    const long long tc = i >> 6;
    const int c = (int)(tc % KC), t = (int)(tc / KC);
    const uint8_t* src = m ? a.w3 : a.w1;
    const int rbase = a.row0 + 16 * t;
    uint8_t v[16];
    if (a.fmt == DSMOE_FMT_FP8) {
      uint8_t* dst = a.w13 + t * tile_b + fp8_w13_chunk_off(c) + m * 512 + l * 16;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        int row, k;
        lane_rows_fp8(l, j, row, k);
        v[j] = src[(long long)(rbase + row) * a.H + 32 * c + k];
      }
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<uint4*>(v);
      if ((c & 7) == 0 && l == 0) {  // the item's scales after its chunks: s1 s1 s3 s3
        const float* s = (const float*)(m ? a.s3 : a.s1);
        const int p = c >> 3, KB = a.H / 128;
        float* sd = reinterpret_cast<float*>(a.w13 + t * tile_b + fp8_w13_scale_off(p, KC));
        for (int h = 0; h < 2; ++h) {
          const int kb = 2 * p + h;
          sd[fp8_w13_scale_index(kb, m)] = kb < KB ? s[(long long)(rbase / 128) * KB + kb] : 0.f;
        }
      }
    } else {
      uint8_t* dst = a.w13 + t * tile_b + (long long)c * 1088 + m * 512 + l * 16;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        int row, k;
        lane_rows_fp4(l, j, row, k);
        const uint8_t* rp = src + (long long)(rbase + row) * (a.H / 2);
        v[j] = (uint8_t)(fp4_code(rp, 64 * c + k) | (fp4_code(rp, 64 * c + k + 16) << 4));
      }
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<uint4*>(v);
      if (l < 8) {  // lanes 0..7 write the 4 scale bytes of row pair (g = l, g + 8)
        const uint8_t* s = (const uint8_t*)(m ? a.s3 : a.s1);
        uint8_t* sd = a.w13 + t * tile_b + (long long)c * 1088 + 1024 + m * 32 + 4 * l;
        const int G = a.H / 32;
        sd[0] = s[(long long)(rbase + l) * G + 2 * c];
        sd[1] = s[(long long)(rbase + l) * G + 2 * c + 1];
        sd[2] = s[(long long)(rbase + l + 8) * G + 2 * c];
        sd[3] = s[(long long)(rbase + l + 8) * G + 2 * c + 1];
      }
    }
  }
}

// One thread per (n-tile, chunk, lane) 16-byte output.
__global__ void pack_w2_kernel(PackArgs a) {
  const int NT = a.H / 16;
  const int KC2 = a.fmt == DSMOE_FMT_FP8 ? a.I_loc / 32 : a.I_loc / 64;
  const long long tile_b = w2_tile_bytes(a.fmt, a.I_loc);
  const long long total = (long long)NT * KC2 * 32;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int l = i & 31;
    const long long nc = i >> 5;
    const int c = (int)(nc % KC2), nt = (int)(nc / KC2);
    const int nbase = 16 * nt;
    uint8_t v[16];
    if (a.fmt == DSMOE_FMT_FP8) {
      uint8_t* dst = a.w2d + nt * tile_b + fp8_w2_chunk_off(c) + l * 16;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        int row, k;
        lane_rows_fp8(l, j, row, k);
        v[j] = a.w2[(long long)(nbase + row) * a.I + a.row0 + 32 * c + k];
      }
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<uint4*>(v);
      if (l == 0) {  // one scale per chunk, after the item's chunks; the item's 8 slots padded with 0
        const int KBI = (a.I + 127) / 128;
        float* sd = reinterpret_cast<float*>(a.w2d + nt * tile_b + fp8_w2_scale_off(c >> 3, KC2));
        sd[c & 7] = ((const float*)a.s2)[(long long)(nbase / 128) * KBI + (a.row0 + 32 * c) / 128];
        if (c == KC2 - 1)
          for (int q = (c & 7) + 1; q < 8; ++q) sd[q] = 0.f;
      }
    } else {
      uint8_t* dst = a.w2d + nt * tile_b + (long long)c * 544 + l * 16;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        int row, k;
        lane_rows_fp4(l, j, row, k);
        const uint8_t* rp = a.w2 + (long long)(nbase + row) * (a.I / 2);
        const int kk = a.row0 + 64 * c + k;
        v[j] = (uint8_t)(fp4_code(rp, kk) | (fp4_code(rp, kk + 16) << 4));
      }
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<uint4*>(v);
      if (l < 8) {
        const uint8_t* s = (const uint8_t*)a.s2;
        uint8_t* sd = a.w2d + nt * tile_b + (long long)c * 544 + 512 + 4 * l;
        const int G = a.I / 32, g0 = (a.row0 + 64 * c) / 32;
        sd[0] = s[(long long)(nbase + l) * G + g0];
        sd[1] = s[(long long)(nbase + l) * G + g0 + 1];
        sd[2] = s[(long long)(nbase + l + 8) * G + g0];
        sd[3] = s[(long long)(nbase + l + 8) * G + g0 + 1];
      }
    }
  }
}

struct UnpackArgs {
  int fmt, H, I, row0, I_loc;
  const uint8_t *w13, *w2s;
  float *w1, *w3, *w2;
};

// Inverse maps, dequantizing with the same conversions the GEMV kernels use.
__global__ void unpack_w13_kernel(UnpackArgs a) {
  const int T = a.I_loc / 16;
  const int KC = a.fmt == DSMOE_FMT_FP8 ? a.H / 32 : a.H / 64;
  const long long tile_b = w13_tile_bytes(a.fmt, a.H);
  const long long total = (long long)T * KC * 2 * 32;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int l = i & 31, m = (i >> 5) & 1;
    const long long tc = i >> 6;
    const int c = (int)(tc % KC), t = (int)(tc / KC);
    float* dst = m ? a.w3 : a.w1;
    const uint8_t* tile = a.w13 + t * tile_b;
    if (a.fmt == DSMOE_FMT_FP8) {
      const uint4 q = ld16(tile + fp8_w13_chunk_off(c) + m * 512 + l * 16);
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
      const float s = reinterpret_cast<const float*>(tile + fp8_w13_scale_off(c >> 3, KC))[fp8_w13_scale_index((32 * c) / 128, m)];
#pragma unroll
      for (int p = 0; p < 8; ++p) {  // p-th byte pair
        const uint32_t h = e4m3x2_to_f16x2((w[p >> 1] >> (16 * (p & 1))) & 0xFFFF);
        int row, k;
        lane_rows_fp8(l, 2 * p, row, k);
        float* o = dst + (long long)(16 * t + row) * a.H + 32 * c + k;
        o[0] = f16_lo(h) * s;
        o[1] = f16_hi(h) * s;
      }
    } else {
      const uint4 q = ld16(tile + (long long)c * 1088 + m * 512 + l * 16);
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
      const uint8_t* sc = tile + (long long)c * 1088 + 1024 + m * 32;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const uint32_t h = e2m1x2_to_f16x2((w[j >> 2] >> (8 * (j & 3))) & 0xFF);
        int row, k;
        lane_rows_fp4(l, j, row, k);
        const int g = row & 7, hi_row = row >> 3, grp = k >> 5;  // group within chunk (0/1)
        const float s = e8m0_to_f32(sc[4 * g + 2 * hi_row + grp]);
        float* o = dst + (long long)(16 * t + row) * a.H + 64 * c + k;
        o[0] = f16_lo(h) * s;   // low nibble: K
        o[16] = f16_hi(h) * s;  // high nibble: K + 16 (same 32-K scale group)
      }
    }
  }
}

__global__ void unpack_w2_kernel(UnpackArgs a) {
  const int NT = a.H / 16;
  const int KC2 = a.fmt == DSMOE_FMT_FP8 ? a.I_loc / 32 : a.I_loc / 64;
  const long long tile_b = w2_tile_bytes(a.fmt, a.I_loc);
  const long long total = (long long)NT * KC2 * 32;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int l = i & 31;
    const long long nc = i >> 5;
    const int c = (int)(nc % KC2), nt = (int)(nc / KC2);
    const uint8_t* tile = a.w2s + nt * tile_b;
    if (a.fmt == DSMOE_FMT_FP8) {
      const uint4 q = ld16(tile + fp8_w2_chunk_off(c) + l * 16);
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
      const float s = reinterpret_cast<const float*>(tile + fp8_w2_scale_off(c >> 3, KC2))[c & 7];
#pragma unroll
      for (int p = 0; p < 8; ++p) {
        const uint32_t h = e4m3x2_to_f16x2((w[p >> 1] >> (16 * (p & 1))) & 0xFFFF);
        int row, k;
        lane_rows_fp8(l, 2 * p, row, k);
        float* o = a.w2 + (long long)(16 * nt + row) * a.I_loc + 32 * c + k;
        o[0] = f16_lo(h) * s;
        o[1] = f16_hi(h) * s;
      }
    } else {
      const uint4 q = ld16(tile + (long long)c * 544 + l * 16);
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
      const uint8_t* sc = tile + (long long)c * 544 + 512;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const uint32_t h = e2m1x2_to_f16x2((w[j >> 2] >> (8 * (j & 3))) & 0xFF);
        int row, k;
        lane_rows_fp4(l, j, row, k);
        const int g = row & 7, hi_row = row >> 3, grp = k >> 5;
        const float s = e8m0_to_f32(sc[4 * g + 2 * hi_row + grp]);
        float* o = a.w2 + (long long)(16 * nt + row) * a.I_loc + 64 * c + k;
        o[0] = f16_lo(h) * s;
        o[16] = f16_hi(h) * s;
      }
    }
  }
}

static int check_geometry(int fmt, int H, int I, int row0, int I_loc) {
  DSMOE_REQUIRE(fmt == DSMOE_FMT_FP8 || fmt == DSMOE_FMT_FP4, DSMOE_ERR_ARG, "store: unknown format %d", fmt);
  DSMOE_REQUIRE(H > 0 && H % 128 == 0, DSMOE_ERR_ARG, "store: hidden %d must be a multiple of 128", H);
  const int kq = fmt == DSMOE_FMT_FP8 ? 32 : 64;
  DSMOE_REQUIRE(I_loc > 0 && I_loc % kq == 0, DSMOE_ERR_ARG,
                "store: inter_local %d must be a multiple of %d for this format", I_loc, kq);
  DSMOE_REQUIRE(row0 >= 0 && row0 % 32 == 0 && row0 + I_loc <= I, DSMOE_ERR_ARG,
                "store: slice [%d, %d) must start on a multiple of 32 and fit in inter %d", row0, row0 + I_loc, I);
  DSMOE_REQUIRE(fmt == DSMOE_FMT_FP8 || I % 32 == 0, DSMOE_ERR_ARG, "store: FP4 inter %d must be a multiple of 32", I);
  return DSMOE_OK;
}

static int grid_cap() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms * 8;
}

}  // namespace dsmoe

using namespace dsmoe;

extern "C" int dsmoe_store_expert_bytes(int fmt, int hidden, int inter_local, long long* w13_bytes,
                                        long long* w2_bytes) {
  DSMOE_REQUIRE(w13_bytes && w2_bytes, DSMOE_ERR_ARG, "store_expert_bytes: null pointer");
  const int rc = check_geometry(fmt, hidden, inter_local, 0, inter_local);
  if (rc) return rc;
  *w13_bytes = (long long)(inter_local / 16) * w13_tile_bytes(fmt, hidden);
  *w2_bytes = (long long)(hidden / 16) * w2_tile_bytes(fmt, inter_local);
  return DSMOE_OK;
}

extern "C" int dsmoe_store_pack_expert(int fmt, int hidden, int inter, int row0, int inter_local,
                                       const uint8_t* w1, const void* s1, const uint8_t* w3, const void* s3,
                                       const uint8_t* w2, const void* s2, uint8_t* w13_dst, uint8_t* w2_dst,
                                       void* stream) {
  int rc = check_geometry(fmt, hidden, inter, row0, inter_local);
  if (rc) return rc;
  DSMOE_REQUIRE(w1 && s1 && w3 && s3 && w2 && s2 && w13_dst && w2_dst, DSMOE_ERR_ARG, "pack_expert: null pointer");
  DSMOE_REQUIRE(((uintptr_t)w13_dst & 15) == 0 && ((uintptr_t)w2_dst & 15) == 0, DSMOE_ERR_ALIGN,
                "pack_expert: destinations must be 16-byte aligned");
  PackArgs a{fmt, hidden, inter, row0, inter_local, w1, w3, w2, s1, s3, s2, w13_dst, w2_dst};
  cudaStream_t st = (cudaStream_t)stream;
  const int cap = grid_cap();
  const long long n13 = (long long)(inter_local / 16) * (fmt == DSMOE_FMT_FP8 ? hidden / 32 : hidden / 64) * 64;
  const long long n2 = (long long)(hidden / 16) * (fmt == DSMOE_FMT_FP8 ? inter_local / 32 : inter_local / 64) * 32;
  pack_w13_kernel<<<(int)std::min<long long>((n13 + 255) / 256, cap), 256, 0, st>>>(a);
  pack_w2_kernel<<<(int)std::min<long long>((n2 + 255) / 256, cap), 256, 0, st>>>(a);
  return cuda_status("pack_expert");
}

extern "C" int dsmoe_store_unpack_expert(int fmt, int hidden, int inter, int row0, int inter_local,
                                         const uint8_t* w13_src, const uint8_t* w2_src, float* w1, float* w3,
                                         float* w2, void* stream) {
  int rc = check_geometry(fmt, hidden, inter, row0, inter_local);
  if (rc) return rc;
  DSMOE_REQUIRE(w13_src && w2_src && w1 && w3 && w2, DSMOE_ERR_ARG, "unpack_expert: null pointer");
  UnpackArgs a{fmt, hidden, inter, row0, inter_local, w13_src, w2_src, w1, w3, w2};
  cudaStream_t st = (cudaStream_t)stream;
  const int cap = grid_cap();
  const long long n13 = (long long)(inter_local / 16) * (fmt == DSMOE_FMT_FP8 ? hidden / 32 : hidden / 64) * 64;
  const long long n2 = (long long)(hidden / 16) * (fmt == DSMOE_FMT_FP8 ? inter_local / 32 : inter_local / 64) * 32;
  unpack_w13_kernel<<<(int)std::min<long long>((n13 + 255) / 256, cap), 256, 0, st>>>(a);
  unpack_w2_kernel<<<(int)std::min<long long>((n2 + 255) / 256, cap), 256, 0, st>>>(a);
  return cuda_status("unpack_expert");
}
