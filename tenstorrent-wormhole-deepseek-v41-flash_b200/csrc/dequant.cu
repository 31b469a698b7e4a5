// Reference-layout unpack kernels and activation quant (the kernel.py operator surface).
//
//   dsmoe_fp8_block_dequant  <- _deq_fp8_weight   (dsv41/ref/kernel.py:75-78)
//   dsmoe_fp4_dequant        <- dequant_fp4_weight (dsv41/ref/kernel.py:91-98), fp4lib dequant_fp4
//                               (dsv41/ref/fp4lib.c:12-30)
//   dsmoe_act_quant          <- act_quant's quantizing branch (dsv41/ref/kernel.py:44-55)
//
// These are HBM-bound byte kernels: each thread turns one 16-byte load of codes into 16 (FP8) or
// 32 (FP4) outputs written with 16-byte stores; grids are a multiple of the SM count.
#include "common.cuh"

namespace dsmoe {

template <typename T>
__device__ __forceinline__ void store4(T* dst, float a, float b, float c, float d);
template <>
__device__ __forceinline__ void store4<float>(float* dst, float a, float b, float c, float d) {
  *reinterpret_cast<float4*>(dst) = make_float4(a, b, c, d);
}
template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16* dst, float a, float b, float c, float d) {
  __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
  uint2 v;
  v.x = *reinterpret_cast<uint32_t*>(&lo);
  v.y = *reinterpret_cast<uint32_t*>(&hi);
  *reinterpret_cast<uint2*>(dst) = v;
}

// One thread per 4 consecutive codes of a row (K % 4 == 0 required by the host check).
template <typename T>
__global__ void fp8_block_dequant_kernel(const uint8_t* __restrict__ b, const float* __restrict__ bs,
                                         long long N, long long K, int block, long long KS,
                                         T* __restrict__ out) {
  const long long n4 = N * (K / 4);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / (K / 4), k = (i % (K / 4)) * 4;
    const uint32_t w = *reinterpret_cast<const uint32_t*>(b + row * K + k);
    const float s = bs[(row / block) * KS + k / block];
    const uint32_t lo = e4m3x2_to_f16x2(w & 0xFFFF), hi = e4m3x2_to_f16x2(w >> 16);
    store4<T>(out + row * K + k, f16_lo(lo) * s, f16_hi(lo) * s, f16_lo(hi) * s, f16_hi(hi) * s);
  }
}

// One thread per 16 packed bytes = 32 values = exactly one e8m0 group (K % 32 == 0).
template <typename T>
__global__ void fp4_dequant_kernel(const uint8_t* __restrict__ b, const uint8_t* __restrict__ bs,
                                   long long N, long long K, T* __restrict__ out) {
  const long long groups = N * (K / 32);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < groups;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / (K / 32), g = i % (K / 32);
    const uint4 q = ld16(b + row * (K / 2) + g * 16);
    const float s = e8m0_to_f32(bs[row * (K / 32) + g]);
    T* o = out + row * K + g * 32;
    const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint32_t h0 = e2m1x2_to_f16x2(words[w] & 0xFF), h1 = e2m1x2_to_f16x2((words[w] >> 8) & 0xFF);
      const uint32_t h2 = e2m1x2_to_f16x2((words[w] >> 16) & 0xFF), h3 = e2m1x2_to_f16x2(words[w] >> 24);
      store4<T>(o + w * 8, f16_lo(h0) * s, f16_hi(h0) * s, f16_lo(h1) * s, f16_hi(h1) * s);
      store4<T>(o + w * 8 + 4, f16_lo(h2) * s, f16_hi(h2) * s, f16_lo(h3) * s, f16_hi(h3) * s);
    }
  }
}

// float -> e4m3 code with round-to-nearest-even and saturation at +-448 (input pre-clamped).
__device__ __forceinline__ uint8_t f32_to_e4m3(float v) {
  unsigned short r;
  asm("{\n\t.reg .b16 t;\n\tcvt.rn.satfinite.e4m3x2.f32 t, %1, %2;\n\tmov.b16 %0, t;\n\t}"
      : "=h"(r) : "f"(0.0f), "f"(v));
  return (uint8_t)(r & 0xFF);
}

// One warp per (row, block of `block` values).
template <typename TI>
__global__ void act_quant_kernel(const TI* __restrict__ x, long long M, long long K, int block, int pow2,
                                 uint8_t* __restrict__ q, float* __restrict__ s) {
  const int lane = threadIdx.x & 31;
  const long long nb = K / block;
  const long long wid = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long item = wid; item < M * nb; item += nw) {
    const long long row = item / nb, blk = item % nb;
    const TI* xr = x + row * K + blk * block;
    float amax = 0.f;
    for (int i = lane; i < block; i += 32) amax = fmaxf(amax, fabsf((float)xr[i]));
    amax = warp_max(amax);
    amax = fmaxf(amax, 1e-4f);
    float sc = amax / 448.0f;
    if (pow2) {
      int e;
      const float m = frexpf(sc, &e);
      sc = ldexpf(1.0f, m == 0.5f ? e - 1 : e);
    }
    if (lane == 0) s[row * nb + blk] = sc;
    for (int i = lane; i < block; i += 32) {
      const float v = fminf(fmaxf((float)xr[i] / sc, -448.0f), 448.0f);
      q[row * K + blk * block + i] = f32_to_e4m3(v);
    }
  }
}

static int grid_for(long long items, int threads) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  long long g = (items + threads - 1) / threads;
  const long long cap = (long long)sms * 16;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace dsmoe

using namespace dsmoe;

extern "C" int dsmoe_fp8_block_dequant(const uint8_t* b, const float* b_s, long long N, long long K,
                                       int block, void* out, int out_dtype, void* stream) {
  DSMOE_REQUIRE(b && b_s && out, DSMOE_ERR_ARG, "fp8_block_dequant: null pointer");
  DSMOE_REQUIRE(N > 0 && K > 0 && K % 4 == 0 && block > 0 && block % 4 == 0, DSMOE_ERR_ARG,
                "fp8_block_dequant: need K %% 4 == 0 and block %% 4 == 0 (N=%lld K=%lld block=%d)", N, K, block);
  DSMOE_REQUIRE(((uintptr_t)b & 3) == 0 && ((uintptr_t)out & 15) == 0, DSMOE_ERR_ALIGN,
                "fp8_block_dequant: misaligned pointer");
  const long long KS = (K + block - 1) / block;
  cudaStream_t st = (cudaStream_t)stream;
  const int threads = 256, grid = grid_for(N * (K / 4), threads);
  if (out_dtype == DSMOE_DTYPE_F32)
    fp8_block_dequant_kernel<float><<<grid, threads, 0, st>>>(b, b_s, N, K, block, KS, (float*)out);
  else if (out_dtype == DSMOE_DTYPE_BF16)
    fp8_block_dequant_kernel<__nv_bfloat16><<<grid, threads, 0, st>>>(b, b_s, N, K, block, KS, (__nv_bfloat16*)out);
  else
    DSMOE_REQUIRE(false, DSMOE_ERR_ARG, "fp8_block_dequant: out_dtype %d", out_dtype);
  return cuda_status("fp8_block_dequant");
}

extern "C" int dsmoe_fp4_dequant(const uint8_t* b, const uint8_t* b_s, long long N, long long K,
                                 void* out, int out_dtype, void* stream) {
  DSMOE_REQUIRE(b && b_s && out, DSMOE_ERR_ARG, "fp4_dequant: null pointer");
  DSMOE_REQUIRE(N > 0 && K > 0 && K % 32 == 0, DSMOE_ERR_ARG, "fp4_dequant: need K %% 32 == 0 (K=%lld)", K);
  DSMOE_REQUIRE(((uintptr_t)b & 15) == 0 && ((uintptr_t)out & 15) == 0, DSMOE_ERR_ALIGN,
                "fp4_dequant: misaligned pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const int threads = 256, grid = grid_for(N * (K / 32), threads);
  if (out_dtype == DSMOE_DTYPE_F32)
    fp4_dequant_kernel<float><<<grid, threads, 0, st>>>(b, b_s, N, K, (float*)out);
  else if (out_dtype == DSMOE_DTYPE_BF16)
    fp4_dequant_kernel<__nv_bfloat16><<<grid, threads, 0, st>>>(b, b_s, N, K, (__nv_bfloat16*)out);
  else
    DSMOE_REQUIRE(false, DSMOE_ERR_ARG, "fp4_dequant: out_dtype %d", out_dtype);
  return cuda_status("fp4_dequant");
}

extern "C" int dsmoe_act_quant(const void* x, int x_dtype, long long M, long long K, int block, int pow2,
                               uint8_t* q, float* s, void* stream) {
  DSMOE_REQUIRE(x && q && s, DSMOE_ERR_ARG, "act_quant: null pointer");
  DSMOE_REQUIRE(M > 0 && K > 0 && block > 0 && K % block == 0, DSMOE_ERR_ARG,
                "act_quant: K (%lld) must be a multiple of block (%d)", K, block);
  cudaStream_t st = (cudaStream_t)stream;
  const int threads = 256, grid = grid_for(M * (K / block) * 32, threads);
  if (x_dtype == DSMOE_DTYPE_F32)
    act_quant_kernel<float><<<grid, threads, 0, st>>>((const float*)x, M, K, block, pow2, q, s);
  else if (x_dtype == DSMOE_DTYPE_BF16)
    act_quant_kernel<__nv_bfloat16><<<grid, threads, 0, st>>>((const __nv_bfloat16*)x, M, K, block, pow2, q, s);
  else
    DSMOE_REQUIRE(false, DSMOE_ERR_ARG, "act_quant: x_dtype %d", x_dtype);
  return cuda_status("act_quant");
}

