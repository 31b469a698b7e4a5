// Kernel-surface GEMMs on block-scaled weights in the reference (checkpoint) layout:
//   dsmoe_fp8_gemm  <- fp8_gemm (dsv41/ref/kernel.py:105-107)
//   dsmoe_fp4_gemm  <- fp4_gemm (dsv41/ref/kernel.py:110-112)
// out = (a * a_s) @ (b * b_s)^T with fp32 accumulation, rounded once to the output dtype.
//
// These serve callers of the reference's operator module (DeepSeek's model.py imports them by
// name); the MoE hot path itself runs on the packed store (moe_decode.cu). Tiles: 64 weight rows x
// 32 tokens per CTA, K in blocks of 128 staged through shared memory; weights widened exactly to
// bf16, activations bf16 (fp32 activations are split into bf16 hi + lo, two MMAs), bf16 tensor-core
// MMA with fp32 accumulation; the fp32 weight scale (FP8, per 128x128) times the activation scale
// (per token and 128-K block) is applied to each block's fp32 partial; FP4's e8m0 scales per 32.
#include "common.cuh"

namespace dsmoe {

constexpr int GM = 64;   // weight rows per CTA (16 per warp)
constexpr int GT = 32;   // tokens per CTA
constexpr int GK = 128;  // K per stage
constexpr int WROW = GK + 16;      // FP8 smem row stride (bytes)
constexpr int WROW4 = GK / 2 + 16; // FP4 smem row stride (bytes)
constexpr int AROW = GK + 8;       // activation smem row stride (bf16 elements)

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t f16x2_to_bf16x2(uint32_t h) {
  __nv_bfloat162 b = __floats2bfloat162_rn(f16_lo(h), f16_hi(h));  // exact for e4m3 / e2m1 values
  return *reinterpret_cast<uint32_t*>(&b);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&b);
}

__device__ __forceinline__ float act_value(const void* a, int dt, long long i) {
  if (dt == DSMOE_DTYPE_F32) return reinterpret_cast<const float*>(a)[i];
  if (dt == DSMOE_DTYPE_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a)[i]);
  const uint32_t h = e4m3x2_to_f16x2(reinterpret_cast<const uint8_t*>(a)[i]);
  return f16_lo(h);
}

template <int FMT>
__global__ void __launch_bounds__(128) block_gemm_kernel(const void* __restrict__ a, int a_dtype,
                                                         const float* __restrict__ a_s, int M, int K,
                                                         const uint8_t* __restrict__ b, const void* __restrict__ b_s,
                                                         int N, void* __restrict__ out, int out_dtype) {
  __shared__ __align__(16) uint8_t wsm[GM * WROW];
  __shared__ __align__(16) uint8_t ssm[GM * 4];
  __shared__ __align__(16) __nv_bfloat16 ahi[GT * AROW];
  __shared__ __align__(16) __nv_bfloat16 alo[GT * AROW];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
  const int n0 = blockIdx.x * GM, m0 = blockIdx.y * GT;
  const bool split = a_dtype == DSMOE_DTYPE_F32;
  const int KB = K / GK;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  for (int kb = 0; kb < KB; ++kb) {
    // stage weights
    if (FMT == DSMOE_FMT_FP8) {
      for (int i = threadIdx.x; i < GM * (GK / 16); i += blockDim.x) {
        const int r = i / (GK / 16), c = i % (GK / 16);
        uint4 v = make_uint4(0, 0, 0, 0);
        if (n0 + r < N) v = ld16(b + (long long)(n0 + r) * K + kb * GK + c * 16);
        *reinterpret_cast<uint4*>(wsm + r * WROW + c * 16) = v;
      }
    } else {
      for (int i = threadIdx.x; i < GM * (GK / 32); i += blockDim.x) {
        const int r = i / (GK / 32), c = i % (GK / 32);
        uint4 v = make_uint4(0, 0, 0, 0);
        if (n0 + r < N) v = ld16(b + (long long)(n0 + r) * (K / 2) + kb * (GK / 2) + c * 16);
        *reinterpret_cast<uint4*>(wsm + r * WROW4 + c * 16) = v;
      }
      for (int i = threadIdx.x; i < GM; i += blockDim.x) {
        uint32_t v = 0x7F7F7F7Fu;
        if (n0 + i < N) v = *reinterpret_cast<const uint32_t*>((const uint8_t*)b_s + (long long)(n0 + i) * (K / 32) + kb * 4);
        *reinterpret_cast<uint32_t*>(ssm + i * 4) = v;
      }
    }
    // stage activations (bf16 hi, and lo for fp32 input)
    for (int i = threadIdx.x; i < GT * GK; i += blockDim.x) {
      const int tkn = i / GK, k = i % GK;
      float v = 0.f;
      if (m0 + tkn < M) v = act_value(a, a_dtype, (long long)(m0 + tkn) * K + kb * GK + k);
      const __nv_bfloat16 h = __float2bfloat16_rn(v);
      ahi[tkn * AROW + k] = h;
      if (split) alo[tkn * AROW + k] = __float2bfloat16_rn(v - __bfloat162float(h));
    }
    __syncthreads();

    float t[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) t[i][j] = 0.f;
    const int r0 = warp * 16 + g;
#pragma unroll
    for (int ks = 0; ks < GK / 16; ++ks) {
      uint32_t A[4];
      const int kk = ks * 16 + 2 * tq;
      if (FMT == DSMOE_FMT_FP8) {
        const uint8_t* w0 = wsm + r0 * WROW;
        const uint8_t* w8 = wsm + (r0 + 8) * WROW;
        A[0] = f16x2_to_bf16x2(e4m3x2_to_f16x2(*reinterpret_cast<const uint16_t*>(w0 + kk)));
        A[1] = f16x2_to_bf16x2(e4m3x2_to_f16x2(*reinterpret_cast<const uint16_t*>(w8 + kk)));
        A[2] = f16x2_to_bf16x2(e4m3x2_to_f16x2(*reinterpret_cast<const uint16_t*>(w0 + kk + 8)));
        A[3] = f16x2_to_bf16x2(e4m3x2_to_f16x2(*reinterpret_cast<const uint16_t*>(w8 + kk + 8)));
      } else {
        const uint8_t* w0 = wsm + r0 * WROW4;
        const uint8_t* w8 = wsm + (r0 + 8) * WROW4;
        A[0] = f16x2_to_bf16x2(e2m1x2_to_f16x2(w0[kk / 2]));
        A[1] = f16x2_to_bf16x2(e2m1x2_to_f16x2(w8[kk / 2]));
        A[2] = f16x2_to_bf16x2(e2m1x2_to_f16x2(w0[kk / 2 + 4]));
        A[3] = f16x2_to_bf16x2(e2m1x2_to_f16x2(w8[kk / 2 + 4]));
      }
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const __nv_bfloat16* ar = ahi + (nt * 8 + g) * AROW + kk;
        mma_bf16(t[nt], A, *reinterpret_cast<const uint32_t*>(ar), *reinterpret_cast<const uint32_t*>(ar + 8));
        if (split) {
          const __nv_bfloat16* al2 = alo + (nt * 8 + g) * AROW + kk;
          mma_bf16(t[nt], A, *reinterpret_cast<const uint32_t*>(al2), *reinterpret_cast<const uint32_t*>(al2 + 8));
        }
      }
      if (FMT == DSMOE_FMT_FP4 && (ks & 1)) {  // end of a 32-K group: apply the rows' e8m0 scales
        const int grp = ks >> 1;
        const float slo = e8m0_to_f32(ssm[r0 * 4 + grp]), shi = e8m0_to_f32(ssm[(r0 + 8) * 4 + grp]);
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          const int c0 = m0 + nt * 8 + 2 * tq;
          const float as0 = a_s && c0 < M ? a_s[(long long)c0 * KB + kb] : 1.f;
          const float as1 = a_s && c0 + 1 < M ? a_s[(long long)(c0 + 1) * KB + kb] : 1.f;
          acc[nt][0] = fmaf(t[nt][0], slo * as0, acc[nt][0]);
          acc[nt][1] = fmaf(t[nt][1], slo * as1, acc[nt][1]);
          acc[nt][2] = fmaf(t[nt][2], shi * as0, acc[nt][2]);
          acc[nt][3] = fmaf(t[nt][3], shi * as1, acc[nt][3]);
#pragma unroll
          for (int j = 0; j < 4; ++j) t[nt][j] = 0.f;
        }
      }
    }
    if (FMT == DSMOE_FMT_FP8) {
      const int KS = (K + 127) / 128;
      const float bs = n0 < N ? reinterpret_cast<const float*>(b_s)[(long long)(n0 / 128) * KS + kb] : 0.f;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int c0 = m0 + nt * 8 + 2 * tq;
        const float as0 = a_s && c0 < M ? a_s[(long long)c0 * KB + kb] : 1.f;
        const float as1 = a_s && c0 + 1 < M ? a_s[(long long)(c0 + 1) * KB + kb] : 1.f;
        acc[nt][0] = fmaf(t[nt][0], bs * as0, acc[nt][0]);
        acc[nt][1] = fmaf(t[nt][1], bs * as1, acc[nt][1]);
        acc[nt][2] = fmaf(t[nt][2], bs * as0, acc[nt][2]);
        acc[nt][3] = fmaf(t[nt][3], bs * as1, acc[nt][3]);
      }
    }
    __syncthreads();
  }
  // epilogue
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int row = n0 + warp * 16 + g + (q >= 2 ? 8 : 0);
      const int col = m0 + nt * 8 + 2 * tq + (q & 1);
      if (row < N && col < M) {
        const long long o = (long long)col * N + row;
        if (out_dtype == DSMOE_DTYPE_F32)
          reinterpret_cast<float*>(out)[o] = acc[nt][q];
        else
          reinterpret_cast<__nv_bfloat16*>(out)[o] = __float2bfloat16_rn(acc[nt][q]);
      }
    }
  }
}

static int launch_gemm(int fmt, const void* a, int a_dtype, const float* a_s, long long M, long long K,
                       const uint8_t* b, const void* b_s, long long N, void* out, int out_dtype, void* stream) {
  DSMOE_REQUIRE(a && b && b_s && out, DSMOE_ERR_ARG, "gemm: null pointer");
  DSMOE_REQUIRE(M > 0 && N > 0 && K > 0 && K % GK == 0, DSMOE_ERR_ARG, "gemm: K (%lld) must be a multiple of 128", K);
  DSMOE_REQUIRE(M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31), DSMOE_ERR_ARG, "gemm: dimension too large");
  DSMOE_REQUIRE(a_dtype == DSMOE_DTYPE_F32 || a_dtype == DSMOE_DTYPE_BF16 || a_dtype == DSMOE_DTYPE_E4M3, DSMOE_ERR_ARG,
                "gemm: a_dtype %d", a_dtype);
  DSMOE_REQUIRE(out_dtype == DSMOE_DTYPE_F32 || out_dtype == DSMOE_DTYPE_BF16, DSMOE_ERR_ARG, "gemm: out_dtype %d",
                out_dtype);
  DSMOE_REQUIRE(((uintptr_t)b & 15) == 0, DSMOE_ERR_ALIGN, "gemm: b must be 16-byte aligned");
  DSMOE_REQUIRE(fmt == DSMOE_FMT_FP8 || ((uintptr_t)b_s & 3) == 0, DSMOE_ERR_ALIGN, "gemm: FP4 scales must be 4-byte aligned");
  dim3 grid((unsigned)((N + GM - 1) / GM), (unsigned)((M + GT - 1) / GT));
  DSMOE_REQUIRE(grid.y <= 65535, DSMOE_ERR_ARG, "gemm: M too large for one launch");
  cudaStream_t st = (cudaStream_t)stream;
  if (fmt == DSMOE_FMT_FP8)
    block_gemm_kernel<DSMOE_FMT_FP8><<<grid, 128, 0, st>>>(a, a_dtype, a_s, (int)M, (int)K, b, b_s, (int)N, out, out_dtype);
  else
    block_gemm_kernel<DSMOE_FMT_FP4><<<grid, 128, 0, st>>>(a, a_dtype, a_s, (int)M, (int)K, b, b_s, (int)N, out, out_dtype);
  return cuda_status("gemm");
}

}  // namespace dsmoe

using namespace dsmoe;

extern "C" int dsmoe_fp8_gemm(const void* a, int a_dtype, const float* a_s, long long M, long long K, const uint8_t* b,
                              const float* b_s, long long N, void* out, int out_dtype, void* stream) {
  return launch_gemm(DSMOE_FMT_FP8, a, a_dtype, a_s, M, K, b, b_s, N, out, out_dtype, stream);
}

extern "C" int dsmoe_fp4_gemm(const void* a, int a_dtype, const float* a_s, long long M, long long K, const uint8_t* b,
                              const uint8_t* b_s, long long N, void* out, int out_dtype, void* stream) {
  return launch_gemm(DSMOE_FMT_FP4, a, a_dtype, a_s, M, K, b, b_s, N, out, out_dtype, stream);
}
