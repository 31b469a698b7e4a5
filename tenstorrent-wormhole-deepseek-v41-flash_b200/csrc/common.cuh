// Shared device helpers for the B200 MoE expert path (sm_100a).
//
// Number formats (the reference's, kept native in HBM):
//   FP8  e4m3fn weight bytes with one fp32 scale per 128x128 block   (dsv41/ref/kernel.py:75-78)
//   FP4  e2m1 codes, two per byte, LOW nibble first, bit 3 = sign,
//        one e8m0 scale (2^(b-127)) per 32 consecutive K values      (dsv41/ref/kernel.py:91-98,
//                                                                      dsv41/ref/fp4lib.c:12-30)
// Weights enter the tensor cores in their own 8-bit form: mma.sync m16n8k32 with e4m3 operands and
// fp32 accumulation. FP8 bytes are used as they are; an FP4 word becomes two e4m3 words with four
// integer operations (the e2m1 value times 2^-6, exact). The fragment order of the packed store
// (store.cu) is the A-operand register order of that instruction, so one 16-byte load per lane
// yields the A fragments of one (FP8) or two (FP4) MMAs. Activations are split into two e4m3
// terms, hi + lo / 16, that occupy adjacent B columns (about 8 significant bits, exact for bf16
// values in the normal e4m3 range after a power-of-2 pre-scale).
#pragma once
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/dsmoe.h"

namespace dsmoe {

constexpr int kWarp = 32;

// ------------------------------------------------------------------ packed-store geometry
// The store is a sequence of work items, each one contiguous run of bytes that carries its own
// scales, so that one bulk copy brings everything an item needs.
// FP8 w1|w3 tile (16 rows of w1 and the same 16 rows of w3): items of 8 chunks of 32 K
// (chunk = w1 512 B + w3 512 B), each followed by its 16 B of fp32 scales
// [s1 block 0, s1 block 1, s3 block 0, s3 block 1] (blocks of 128 K); the last item may be short.
// FP8 w2 n-tile (16 output rows): items of 8 chunks of 32 K (512 B each) followed by 32 B holding
// one fp32 scale per chunk.
// FP4 w1|w3 tile: H/64 chunks of 1088 B (w1 512, w3 512, w1 scales 32, w3 scales 32).
// FP4 w2 n-tile: I_loc/64 chunks of 544 B (512 data, 32 scales).
constexpr int kFp8W13Item = 8 * 1024 + 16;
constexpr int kFp8W2Item = 8 * 512 + 32;

__host__ __device__ inline long long fp8_w13_chunk_off(int c) { return (long long)(c >> 3) * kFp8W13Item + (c & 7) * 1024; }
__host__ __device__ inline long long fp8_w13_scale_off(int p, int KC) {
  const int n = KC - 8 * p;
  return (long long)p * kFp8W13Item + (n < 8 ? n : 8) * 1024;
}
// index (in floats) of the scale of 128-K block `kb` of matrix m (0 = w1, 1 = w3) within its item
__host__ __device__ inline int fp8_w13_scale_index(int kb, int m) { return 2 * m + (kb & 1); }
__host__ __device__ inline long long fp8_w2_chunk_off(int c) { return (long long)(c >> 3) * kFp8W2Item + (c & 7) * 512; }
__host__ __device__ inline long long fp8_w2_scale_off(int p, int KC2) {
  const int n = KC2 - 8 * p;
  return (long long)p * kFp8W2Item + (n < 8 ? n : 8) * 512;
}

__host__ __device__ inline long long fp8_w13_tile_bytes(int H) {
  const int KC = H / 32;
  return (long long)(KC / 8) * kFp8W13Item + (KC % 8 ? (KC % 8) * 1024 + 16 : 0);
}
__host__ __device__ inline long long fp8_w2_tile_bytes(int I_loc) {
  const int KC2 = I_loc / 32;
  return (long long)(KC2 / 8) * kFp8W2Item + (KC2 % 8 ? (KC2 % 8) * 512 + 32 : 0);
}
__host__ __device__ inline long long fp4_w13_tile_bytes(int H) { return (long long)(H / 64) * 1088; }
__host__ __device__ inline long long fp4_w2_tile_bytes(int I_loc) { return (long long)(I_loc / 64) * 544; }

__host__ __device__ inline long long w13_tile_bytes(int fmt, int H) {
  return fmt == DSMOE_FMT_FP8 ? fp8_w13_tile_bytes(H) : fp4_w13_tile_bytes(H);
}
__host__ __device__ inline long long w2_tile_bytes(int fmt, int I_loc) {
  return fmt == DSMOE_FMT_FP8 ? fp8_w2_tile_bytes(I_loc) : fp4_w2_tile_bytes(I_loc);
}

// ------------------------------------------------------------------ number conversions
// Two e4m3 codes (low byte = first element) -> f16x2 (low half = first element). Exact.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t two_bytes) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"((unsigned short)two_bytes));
  return r;
}

// One byte holding two e2m1 codes (low nibble = first element) -> f16x2. Exact.
__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t byte) {
  uint32_t r;
  asm("{\n\t.reg .b8 t;\n\tcvt.u8.u32 t, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, t;\n\t}" : "=r"(r) : "r"(byte));
  return r;
}

// e8m0 byte -> 2^(b-127) as fp32. b = 0 is the subnormal 2^-127; 0xFF is NaN (torch semantics).
__device__ __forceinline__ float e8m0_to_f32(uint32_t b) {
  b &= 0xFFu;
  const uint32_t bits = b == 0u ? 0x00400000u : (b == 0xFFu ? 0x7FC00000u : b << 23);
  return __uint_as_float(bits);
}

// Four e8m0 bytes -> 2^(b-127) each. Byte shifts into the fp32 exponent field; the two codes
// that are not plain powers of two (0 -> 2^-127, 0xFF -> NaN) take the exact per-byte path.
__device__ __forceinline__ void e8m0x4_to_f32(uint32_t sv, float& s0, float& s1, float& s2, float& s3) {
  s0 = __uint_as_float((sv & 0xFFu) << 23);
  s1 = __uint_as_float((sv & 0xFF00u) << 15);
  s2 = __uint_as_float((sv & 0xFF0000u) << 7);
  s3 = __uint_as_float((sv >> 1) & 0x7F800000u);
  const uint32_t zero_or_ff = (((sv - 0x01010101u) & ~sv) | ((~sv - 0x01010101u) & sv)) & 0x80808080u;
  if (zero_or_ff) {
    s0 = e8m0_to_f32(sv);
    s1 = e8m0_to_f32(sv >> 8);
    s2 = e8m0_to_f32(sv >> 16);
    s3 = e8m0_to_f32(sv >> 24);
  }
}

__device__ __forceinline__ float f16_lo(uint32_t h2) { return __half2float(__ushort_as_half((unsigned short)(h2 & 0xFFFF))); }
__device__ __forceinline__ float f16_hi(uint32_t h2) { return __half2float(__ushort_as_half((unsigned short)(h2 >> 16))); }

// ------------------------------------------------------------------ 8-bit tensor-core path
// D += A(16x32, e4m3, row) * B(32x8, e4m3, col), fp32 accumulate. A registers: a0 = row g, K 4t..4t+3;
// a1 = row g+8; a2 = row g, K 16+4t..; a3 = row g+8, K 16+4t.. (g = lane/4, t = lane%4).
// B registers: b0 = K 4t..4t+3 of column g, b1 = K 16+4t.. of column g.
__device__ __forceinline__ void mma_e4m3(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D = A * B with C = 0 (a fresh partial that the caller scales).
__device__ __forceinline__ void mma_e4m3_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.0f));
}

// One 32-bit word of packed FP4 (four bytes, two e2m1 codes each, bit 3 of a code = sign) ->
// two words of e4m3: `lo` from the low nibbles, `hi` from the high nibbles. The e4m3 byte
// ((code & 7) << 2) | ((code & 8) << 4) equals the e2m1 value times 2^-6 for all 16 codes (the
// 2^6 is applied with the group scale), so this is exact and needs no conversion instruction.
__device__ __forceinline__ void fp4w_to_e4m3(uint32_t w, uint32_t& lo, uint32_t& hi) {
  lo = ((w << 2) & 0x1C1C1C1Cu) | ((w << 4) & 0x80808080u);
  hi = ((w >> 2) & 0x1C1C1C1Cu) | (w & 0x80808080u);
}
constexpr float kFp4E4m3Scale = 64.0f;  // undoes the 2^-6 of fp4w_to_e4m3

// Two fp32 -> two e4m3 (low byte = v0), round to nearest even, saturating at +-448.
__device__ __forceinline__ uint32_t f32x2_to_e4m3x2(float v0, float v1) {
  unsigned short r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(v1), "f"(v0));
  return r;
}
// Activation split for the 8-bit MMA: v ~= hi + lo / kLoScale, two values at a time (low byte =
// v0). hi keeps 4 significant bits, lo the next 4 (|v| <= 448).
constexpr float kLoScale = 16.0f;
constexpr float kLoInv = 1.0f / 16.0f;
__device__ __forceinline__ void split2_e4m3(float v0, float v1, uint32_t& hi2, uint32_t& lo2) {
  hi2 = f32x2_to_e4m3x2(v0, v1);
  const uint32_t b = e4m3x2_to_f16x2(hi2);  // exact
  lo2 = f32x2_to_e4m3x2((v0 - f16_lo(b)) * kLoScale, (v1 - f16_hi(b)) * kLoScale);
}

// One FP4 chunk (64 K: two k32 MMAs, each with its own per-row 32-K group scales) of one matrix
// against NTL n-tiles of activations; fp32 partials scaled and added to acc (times 2^-6, see
// fp4w_to_e4m3). Scale word bytes: (row g, group 0), (g, 1), (g + 8, 0), (g + 8, 1).
template <int NTL>
__device__ __forceinline__ void fp4_chunk_mma(const uint4& w, uint32_t sv, const uint4* xv, float (*acc)[4]) {
  uint32_t l0, h0, l1, h1, l2, h2, l3, h3;
  fp4w_to_e4m3(w.x, l0, h0);
  fp4w_to_e4m3(w.y, l1, h1);
  fp4w_to_e4m3(w.z, l2, h2);
  fp4w_to_e4m3(w.w, l3, h3);
  float sa0, sb0, sa1, sb1;
  e8m0x4_to_f32(sv, sa0, sb0, sa1, sb1);
#pragma unroll
  for (int j = 0; j < NTL; ++j) {
    float d[4], e[4];
    mma_e4m3_z(d, l0, l1, h0, h1, xv[j].x, xv[j].y);
    mma_e4m3_z(e, l2, l3, h2, h3, xv[j].z, xv[j].w);
    acc[j][0] = fmaf(e[0], sb0, fmaf(d[0], sa0, acc[j][0]));
    acc[j][1] = fmaf(e[1], sb0, fmaf(d[1], sa0, acc[j][1]));
    acc[j][2] = fmaf(e[2], sb1, fmaf(d[2], sa1, acc[j][2]));
    acc[j][3] = fmaf(e[3], sb1, fmaf(d[3], sa1, acc[j][3]));
  }
}

// Activation rows (one row per token and term) hold K in the B-operand order of m16n8k32, in blocks
// of 64 K: lane t's 16 bytes at 64 * block + 16 * t are
//   [K 4t..4t+3 | K 16+4t.. | K 32+4t.. | K 48+4t..]   (b0 / b1 of the block's two k32 steps).
__host__ __device__ __forceinline__ int qk_off(int k) {
  return (k >> 6) * 64 + ((k >> 2) & 3) * 16 + ((k >> 5) & 1) * 8 + ((k >> 4) & 1) * 4 + (k & 3);
}

// Streaming 16-byte load of weight data: read once per step, keep it out of L1.
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

__device__ __forceinline__ uint4 ld16(const void* p) { return *reinterpret_cast<const uint4*>(p); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ------------------------------------------------------------------ async copies, mbarriers, bounded waits
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}"
               ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// Wait for the phase of `bar` with parity `parity` to complete; false after `limit_ns`.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_test(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_test(bar, parity)) {
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
  return true;
}
// 1-D bulk copy global -> this CTA's shared memory, completion counted on `bar` (bytes % 16 == 0).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}
// L2 policy for bytes read once per step (expert and router weights): first to be evicted, so the
// kernel's code, tokens and scratch stay resident in L2 across the stream.
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ uint32_t ld_acquire_u32(const unsigned* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// L2-coherent loads of data other CTAs wrote during this launch (skip the non-coherent L1).
__device__ __forceinline__ uint4 ld_cg16(const void* p) {
  uint4 r;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
__device__ __forceinline__ double ld_cg_f64(const double* p) {
  double r;
  asm volatile("ld.global.cg.f64 %0, [%1];" : "=d"(r) : "l"(p));
  return r;
}
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

}  // namespace dsmoe

// ------------------------------------------------------------------ host-side status helpers
namespace dsmoe {
void set_error(const char* fmt, ...);
int cuda_status(const char* where);  // DSMOE_OK or DSMOE_ERR_CUDA after a launch
}  // namespace dsmoe

#define DSMOE_REQUIRE(cond, code, ...)          \
  do {                                          \
    if (!(cond)) {                              \
      ::dsmoe::set_error(__VA_ARGS__);          \
      return (code);                            \
    }                                           \
  } while (0)
