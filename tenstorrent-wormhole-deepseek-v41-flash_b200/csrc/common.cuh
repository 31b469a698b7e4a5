// Shared device helpers for the B200 MoE expert path (sm_100a).
//
// Number formats (the reference's, kept native in HBM):
//   FP8  e4m3fn weight bytes with one fp32 scale per 128x128 block   (dsv41/ref/kernel.py:75-78)
//   FP4  e2m1 codes, two per byte, LOW nibble first, bit 3 = sign,
//        one e8m0 scale (2^(b-127)) per 32 consecutive K values      (dsv41/ref/kernel.py:91-98,
//                                                                      dsv41/ref/fp4lib.c:12-30)
// Weights are widened on the fly to f16 (exact for every e4m3 and e2m1 value) and fed to the
// tensor cores with mma.sync m16n8k16 (f16 x f16 -> fp32). The fragment order of the packed store
// (store.cu) is the A-operand register order of that instruction, so one 16-byte load per lane
// yields the whole A fragment of 2 (FP8) or 4 (FP4) k16 steps.
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

__device__ __forceinline__ float f16_lo(uint32_t h2) { return __half2float(__ushort_as_half((unsigned short)(h2 & 0xFFFF))); }
__device__ __forceinline__ float f16_hi(uint32_t h2) { return __half2float(__ushort_as_half((unsigned short)(h2 >> 16))); }

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// ------------------------------------------------------------------ tensor-core fragment op
// D = A(16x16, f16, row) * B(16x8, f16, col) + C, fp32 accumulate.
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// A fragment of one k16 step from 8 FP8 bytes (two 32-bit words of a lane's packed chunk).
__device__ __forceinline__ void a_frag_fp8(uint32_t (&a)[4], uint32_t w_lo, uint32_t w_hi) {
  a[0] = e4m3x2_to_f16x2(w_lo & 0xFFFF);
  a[1] = e4m3x2_to_f16x2(w_lo >> 16);
  a[2] = e4m3x2_to_f16x2(w_hi & 0xFFFF);
  a[3] = e4m3x2_to_f16x2(w_hi >> 16);
}

// A fragment of one k16 step from 4 FP4 bytes (one 32-bit word of a lane's packed chunk).
__device__ __forceinline__ void a_frag_fp4(uint32_t (&a)[4], uint32_t w) {
  a[0] = e2m1x2_to_f16x2(w & 0xFF);
  a[1] = e2m1x2_to_f16x2((w >> 8) & 0xFF);
  a[2] = e2m1x2_to_f16x2((w >> 16) & 0xFF);
  a[3] = e2m1x2_to_f16x2(w >> 24);
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
