// Kernel-surface GEMMs on block-scaled weights in the reference (checkpoint) layout:
//   dsmoe_fp8_gemm  <- fp8_gemm (dsv41/ref/kernel.py:105-107)
//   dsmoe_fp4_gemm  <- fp4_gemm (dsv41/ref/kernel.py:110-112)
// out[M, N] = (a * a_s per 128-K block) @ dequant(b, b_s)^T with fp32 accumulation, rounded once to
// the output dtype. These serve callers of the reference's operator module (DeepSeek's model.py
// imports them by name for every quantized linear); the MoE hot path itself runs on the resident
// stores.
//
// Two kernels, both on the 5th-generation tensor cores with fp32 accumulators in tensor memory:
// gemm_f8_kernel takes e4m3 activations (act_quant's output) and multiplies the codes as they are
// (further down); gemm_tc_kernel takes fp32 or bf16 activations and converts. In both, one CTA
// computes a tile of 128 weight rows x TT tokens over a range of 128-K blocks.
//
// gemm_tc_kernel (TT = 16, 32 or 64; tcgen05.mma kind::f16, bf16 operands):
//   warp 0      TMA producer: per 128-K block, one tiled load of the raw weight tile (e4m3 bytes, or
//               packed e2m1 bytes) and one of the raw activation tile (fp32 / bf16 / e4m3), rows past
//               N or M read as zero; a ring of RS stages.
//   warps 2-9   converters: weights to bf16, exactly (e4m3 and e2m1 x e8m0 are bf16 values); each
//               activation element times its scales, v = a * a_s[t][kb] * b_s[kb] (b_s only for FP8,
//               whose fp32 scale is one per 128 x 128 block), split into v ~ hi + lo, both bf16
//               (|v - hi - lo| <= 2^-17 |v|). Written in the canonical K-major 128-byte-swizzled
//               layout tcgen05 reads, double-buffered.
//   warp 1      lane 0 issues the MMAs: per 16-K step one MMA over the B tile that holds the hi rows
//               (columns 0..TT-1 of the accumulator) and the lo rows (columns TT..2TT-1), M 128,
//               N 2 TT; warp 1 owns the tensor-memory allocation.
//   warps 2-9   epilogue: tcgen05.ld of the accumulator (two warps per 32-lane quadrant, splitting
//               the tokens), hi column + lo column, coalesced stores of out[token][row].
// Few tiles (small M): the K blocks are split over S CTAs per tile; each writes its fp32 partial to a
// static device array and the last to arrive on the tile's counter sums the S partials in split
// order (deterministic), writes the tile and resets the counter. Calls on one device must therefore
// be ordered (one stream).
// Every wait is bounded; a CTA whose wait expired writes NaN into its share of the output.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace dsmoe {
namespace gemm {

constexpr int NT = 320;                 // 10 warps
constexpr int CT = 256;                 // converting / epilogue threads (warps 2-9)
constexpr int TM = 128;                 // weight rows per tile (MMA M)
constexpr int TTMAX = 64;               // tokens per tile (MMA N)
constexpr int CS = 2;                   // converted stages
constexpr int A_BYTES = TM * 128 * 2;   // bf16 weights of one 128-K block: two 64-K SW128 atoms
constexpr int MAXRS = 4;                // raw stages
constexpr int MAXSLOT = 160;            // split-K partial tiles (static device array)
constexpr int F8TTMAX = 128;            // tokens per tile of the FP8 x e4m3 kernel
constexpr int PART = TM * F8TTMAX;      // floats per partial tile ([col][row])
constexpr uint64_t kWaitNs = 1000000000ull;
constexpr uint32_t TM_COLS = 128;

struct Args {
  CUtensorMap tw;        // weights: {K bytes (FP8) or K/2 bytes (FP4), N}, box {128 | 64, 128}
  CUtensorMap ta;        // activations: {K, M} in a_dtype, box {128, TT}
  const void* b_s;       // FP8: fp32 [ceil(N/128)][K/128]; FP4: e8m0 [N][K/32]
  const float* a_s;      // [M][K/128] or null
  void* out;             // [M][N]
  float* part;           // [MAXSLOT][PART] (S > 1)
  unsigned* cnt;         // [tiles] arrival counters (S > 1), zero between launches
  int M, N, K, TT, tiles_n, tiles, S, nkb, RS, out_f32, lo, w_bytes, a_bytes;
};

__device__ __forceinline__ uint32_t sw128(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void mma_bf16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* tm, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n\t"
               "tcgen05.wait::ld.sync.aligned;"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// 16 / 32 consecutive accumulator columns of this warp's 32 lanes, load and wait in one statement
// (so no use of the registers can be scheduled before the wait).
__device__ __forceinline__ void ld16w(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
               "tcgen05.wait::ld.sync.aligned;"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                 "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
               : "r"(taddr)
               : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void ld32w(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
               "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
               "tcgen05.wait::ld.sync.aligned;"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                 "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
                 "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
                 "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
                 "=r"(r[30]), "=r"(r[31])
               : "r"(taddr)
               : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint32_t bf2(float lo, float hi) {
  __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&b);
}

// Two e4m3 codes -> bf16x2 (exact: every e4m3 value is a bf16 value).
__device__ __forceinline__ uint32_t e4m3x2_to_bf16x2(uint32_t two) {
  const uint32_t h = e4m3x2_to_f16x2(two);
  return bf2(f16_lo(h), f16_hi(h));
}

// Eight activation elements of row t, K offset 8 c within the 128-K block, as fp32.
__device__ __forceinline__ void act8(const uint8_t* raw, int a_dtype, int t, int c, float (&v)[8]) {
  if (a_dtype == DSMOE_DTYPE_F32) {
    const float4* p = reinterpret_cast<const float4*>(raw + (size_t)t * 512 + c * 32);
    const float4 x = p[0], y = p[1];
    v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
    v[4] = y.x; v[5] = y.y; v[6] = y.z; v[7] = y.w;
  } else if (a_dtype == DSMOE_DTYPE_BF16) {
    const uint4 u = *reinterpret_cast<const uint4*>(raw + (size_t)t * 256 + c * 16);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  } else {
    const uint2 u = *reinterpret_cast<const uint2*>(raw + (size_t)t * 128 + c * 8);
    const uint32_t w[2] = {u.x, u.y};
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint32_t h0 = e4m3x2_to_f16x2(w[i] & 0xFFFFu), h1 = e4m3x2_to_f16x2(w[i] >> 16);
      v[4 * i] = f16_lo(h0);
      v[4 * i + 1] = f16_hi(h0);
      v[4 * i + 2] = f16_lo(h1);
      v[4 * i + 3] = f16_hi(h1);
    }
  }
}

template <int FMT, int ADT>
__global__ void __launch_bounds__(NT, 1) gemm_tc_kernel(const __grid_constant__ Args a) {
  extern __shared__ __align__(1024) uint8_t gsm[];
  uint8_t* base = gsm + ((1024 - (smem_u32(gsm) & 1023)) & 1023);
  const int TT = a.TT;
  const int NB = a.lo ? 2 * TT : TT;  // B rows (MMA N): TT hi rows, then TT lo rows
  const int BB = NB * 256;             // one B tile: two 64-K atoms of NB rows x 128 bytes
  uint8_t* sA = base;                                  // [CS][A_BYTES]
  uint8_t* sB = sA + CS * A_BYTES;                     // [CS][BB] (sized for 2 TT rows)
  uint8_t* sR = sB + CS * 2 * TT * 256;                // [RS][w_bytes + a_bytes]
  const int RB = a.w_bytes + a.a_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sR + a.RS * RB);
  uint64_t* rfull = bars;               // [MAXRS] raw stage landed
  uint64_t* rempty = rfull + MAXRS;     // [MAXRS] raw stage read (one arrival per converting warp)
  uint64_t* cfull = rempty + MAXRS;     // [CS] converted stage written (one arrival per converting warp)
  uint64_t* cempty = cfull + CS;        // [CS] MMAs done with the converted stage
  uint64_t* accd = cempty + CS;         // [1] every MMA done
  uint32_t* tslot = reinterpret_cast<uint32_t*>(accd + 1);
  volatile int* abortf = reinterpret_cast<volatile int*>(tslot + 1);
  volatile int* lastf = abortf + 1;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x % a.tiles, z = blockIdx.x / a.tiles;
  const int tn = tile % a.tiles_n, tmi = tile / a.tiles_n;
  const int n0 = tn * TM, m0 = tmi * TT;
  const int kb0 = (int)((long long)z * a.nkb / a.S), kb1 = (int)((long long)(z + 1) * a.nkb / a.S);
  const int nk = kb1 - kb0;

  if (tid == 0) {
    for (int s = 0; s < MAXRS; ++s) {
      mbar_init(&rfull[s], 1);
      mbar_init(&rempty[s], 8);
    }
    for (int s = 0; s < CS; ++s) {
      mbar_init(&cfull[s], 8);
      mbar_init(&cempty[s], 1);
    }
    mbar_init(accd, 1);
    *abortf = 0;
    *lastf = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(TM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tslot;
  auto wait = [&](uint64_t* bar, uint32_t par) -> bool {
    if (*abortf) return false;
    if (!mbar_wait(bar, par, kWaitNs)) {
      *abortf = 1;
      return false;
    }
    return true;
  };

  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(&a.tw) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(&a.ta) : "memory");
      int issued = 0;
      for (int i = 0; i < nk; ++i) {
        const int s = i % a.RS;
        if (i >= a.RS && !wait(&rempty[s], ((i / a.RS) - 1) & 1)) break;
        uint8_t* raw = sR + s * RB;
        const int kb = kb0 + i;
        mbar_expect_tx(&rfull[s], (uint32_t)(a.w_bytes + a.a_bytes));
        tma_2d(raw, &a.tw, FMT == DSMOE_FMT_FP8 ? kb * 128 : kb * 64, n0, &rfull[s]);
        tma_2d(raw + a.w_bytes, &a.ta, kb * 128, m0, &rfull[s]);
        ++issued;
      }
      // every copy issued has landed before the CTA may exit (the last use of each stage)
      for (int i = issued - 1; i >= 0 && i >= issued - a.RS; --i) mbar_wait(&rfull[i % a.RS], (i / a.RS) & 1, kWaitNs);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(NB >> 3) << 17) | ((uint32_t)(TM >> 4) << 24);
      // descriptors of stage 0; another stage, atom or 16-K step moves the start address field
      // (address >> 4): +A_BYTES or +BB per stage, +16384 or +NB*128 per atom, +32 per step
      const uint64_t da0 = desc_sw128(smem_u32(sA)), db0 = desc_sw128(smem_u32(sB));
      const uint64_t bstep = (uint64_t)(NB * 128) >> 4;
      for (int i = 0; i < nk; ++i) {
        const int cs = i % CS;
        if (!wait(&cfull[cs], (i / CS) & 1)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint64_t da = da0 + (uint64_t)(cs * (A_BYTES >> 4)), db = db0 + (uint64_t)(cs * (BB >> 4));
#pragma unroll
        for (int k16 = 0; k16 < 8; ++k16) {
          const uint64_t o = (uint64_t)(k16 & 3) * 2u;
          mma_bf16(tmem, da + (uint64_t)(k16 >> 2) * 1024u + o, db + (uint64_t)(k16 >> 2) * bstep + o, idesc,
                   (i > 0 || k16 > 0) ? 1u : 0u);
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                     ::"r"(smem_u32(&cempty[cs])) : "memory");
      }
      // the accumulator is final (or, after an abort, no MMA is in flight) once this arrives; the
      // tensor memory is freed only after it has
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                   ::"r"(smem_u32(accd)) : "memory");
      mbar_wait(accd, 0, kWaitNs);
    }
  } else {
    // ---------------- converters (warps 2-9), then the epilogue
    const int ct = tid - 64;
    const int c16 = ct & 15;        // this thread's 8-K chunk in every row it converts
    const int rw = ct >> 4;         // first weight row; rows rw + 16 j
    const int nt = TT / 16;         // token rows per thread: rw + 16 j, j < nt
    const int KS = a.K / 128;
    // per-block scales, loaded one block ahead
    float bs_n = 1.f, as_n[4] = {1.f, 1.f, 1.f, 1.f};
    uint32_t ws_n[8] = {127u, 127u, 127u, 127u, 127u, 127u, 127u, 127u};
    auto load_scales = [&](int kb) {
      if (FMT == DSMOE_FMT_FP8) bs_n = reinterpret_cast<const float*>(a.b_s)[(long long)(n0 / 128) * KS + kb];
      if (FMT == DSMOE_FMT_FP4) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int r = n0 + rw + 16 * j;
          ws_n[j] = r < a.N ? reinterpret_cast<const uint8_t*>(a.b_s)[(long long)r * (a.K / 32) + kb * 4 + (c16 >> 2)]
                            : 127u;
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int t = m0 + rw + 16 * j;
        as_n[j] = (a.a_s && j < nt && t < a.M) ? a.a_s[(long long)t * KS + kb] : 1.f;
      }
    };
    if (nk > 0) load_scales(kb0);
    for (int i = 0; i < nk; ++i) {
      const int s = i % a.RS, cs = i % CS;
      const float bs = bs_n;
      float as[4];
      uint32_t wsc[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) as[j] = as_n[j];
#pragma unroll
      for (int j = 0; j < 8; ++j) wsc[j] = ws_n[j];
      if (i + 1 < nk) load_scales(kb0 + i + 1);
      if (!wait(&rfull[s], (i / a.RS) & 1)) break;
      if (i >= CS && !wait(&cempty[cs], ((i / CS) - 1) & 1)) break;
      const uint8_t* raw = sR + s * RB;
      uint8_t* A = sA + cs * A_BYTES;
      uint8_t* Bt = sB + cs * BB;
      const int at = c16 >> 3, cc = c16 & 7;
      // weights: 128 rows x 16 chunks of 8 K
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int r = rw + 16 * j;
        uint4 o;
        if (FMT == DSMOE_FMT_FP8) {
          const uint2 u = *reinterpret_cast<const uint2*>(raw + r * 128 + c16 * 8);
          o = make_uint4(e4m3x2_to_bf16x2(u.x & 0xFFFFu), e4m3x2_to_bf16x2(u.x >> 16), e4m3x2_to_bf16x2(u.y & 0xFFFFu),
                         e4m3x2_to_bf16x2(u.y >> 16));
        } else {
          const uint32_t u = *reinterpret_cast<const uint32_t*>(raw + r * 64 + c16 * 4);
          const float sc = e8m0_to_f32(wsc[j]);
          uint32_t q[4];
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const uint32_t f = e2m1x2_to_f16x2((u >> (8 * h)) & 0xFFu);
            q[h] = bf2(f16_lo(f) * sc, f16_hi(f) * sc);
          }
          o = make_uint4(q[0], q[1], q[2], q[3]);
        }
        *reinterpret_cast<uint4*>(A + at * 16384 + sw128(r, cc)) = o;
      }
      // activations: TT rows x 16 chunks, v = a * a_s * b_s as bf16 hi + lo
      const uint8_t* ra = raw + a.w_bytes;
      for (int j = 0; j < nt; ++j) {
        const int t = rw + 16 * j;
        float v[8];
        act8(ra, ADT, t, c16, v);
        const float sc = as[j] * bs;
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float x0 = v[2 * h] * sc, x1 = v[2 * h + 1] * sc;
          const __nv_bfloat16 b0 = __float2bfloat16_rn(x0), b1 = __float2bfloat16_rn(x1);
          hi[h] = (uint32_t)__bfloat16_as_ushort(b0) | ((uint32_t)__bfloat16_as_ushort(b1) << 16);
          lo[h] = bf2(x0 - __bfloat162float(b0), x1 - __bfloat162float(b1));
        }
        uint8_t* atom = Bt + at * (NB * 128);
        *reinterpret_cast<uint4*>(atom + sw128(t, cc)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        if (a.lo) *reinterpret_cast<uint4*>(atom + sw128(TT + t, cc)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&rempty[s]);
        mbar_arrive(&cfull[cs]);
      }
    }

    // ---------------- epilogue
    const bool landed = mbar_wait(accd, 0, kWaitNs);
    const bool ok = landed && !*abortf;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const int qd = warp & 3, half = (warp - 2) >> 2;
    const int row_l = 32 * qd + lane, row = n0 + row_l;
    const int c0 = half * (TT / 2), nc = TT / 2;
    const uint32_t taddr = tmem + ((uint32_t)(32 * qd) << 16);
    const float nanv = __int_as_float(0x7FC00000);
    auto store = [&](int col, float v) {
      const int t = m0 + col;
      if (row < a.N && t < a.M) {
        const long long o = (long long)t * a.N + row;
        if (a.out_f32) reinterpret_cast<float*>(a.out)[o] = v;
        else reinterpret_cast<__nv_bfloat16*>(a.out)[o] = __float2bfloat16_rn(v);
      }
    };
    // tokens c .. c + 7: hi column plus lo column
    auto load8 = [&](int c, float (&v)[8]) {
      ld8(taddr + (uint32_t)c, v);
      if (a.lo) {
        float w[8];
        ld8(taddr + (uint32_t)(TT + c), w);
#pragma unroll
        for (int q = 0; q < 8; ++q) v[q] += w[q];
      }
    };
    if (a.S == 1) {
      for (int c = c0; c < c0 + nc; c += 8) {
        float v[8];
        load8(c, v);
#pragma unroll
        for (int q = 0; q < 8; ++q) store(c + q, ok ? v[q] : nanv);
      }
    } else {
      float* mine = a.part + (long long)blockIdx.x * PART;
      for (int c = c0; c < c0 + nc; c += 8) {
        float v[8];
        load8(c, v);
#pragma unroll
        for (int q = 0; q < 8; ++q) mine[(c + q) * TM + row_l] = ok ? v[q] : nanv;
      }
      __threadfence();
      named_bar_sync(1, CT);
      if (ct == 0) {
        const unsigned prev = atomicAdd(&a.cnt[tile], 1u);
        *lastf = prev == (unsigned)(a.S - 1);
      }
      named_bar_sync(1, CT);
      if (*lastf) {
        __threadfence();
        for (int c = c0; c < c0 + nc; ++c) {
          float acc = 0.f;
          for (int zz = 0; zz < a.S; ++zz) {
            const float* p = a.part + (long long)(zz * a.tiles + tile) * PART + c * TM + row_l;
            float x;
            asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(x) : "l"(p));
            acc += x;
          }
          store(c, acc);
        }
        if (ct == 0) a.cnt[tile] = 0u;  // ready for the next launch
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TM_COLS) : "memory");
  }
}

// ------------------------------------------------------------------ FP8 / FP4 weights x e4m3 activations
// The fake-quant form model.py passes (act_quant's e4m3 codes + fp32 scale per 128-K block) needs
// no conversion: the TMA lands both operands in the canonical K-major 128-byte-swizzled layout and
// the tensor core multiplies the codes exactly, K 32 per instruction. FP8 weights: kind::f8f6f4.
// FP4 weights: kind::mxf8f6f4.block_scale with A = e2m1 (the TMA widens the packed codes into the
// padded form the tensor core reads) and the checkpoint's e8m0 group scales as A scale factors in
// tensor memory (written two stages ahead by the epilogue warps; B scale factors 1.0). One
// accumulator per 128-K block (a ring of F8ACC in tensor memory); the epilogue warps fold each block
// into fp32 registers with its scales, acc += D * a_s[t][kb] (* b_s[kb] for FP8), while the next
// blocks' MMAs run.
constexpr int F8ACC = 4;
constexpr int F8MAXRS = 10;
constexpr uint32_t F4_SFA = 320, F4_SFB = 416;  // tensor-memory columns of the scale factors (FP4)
constexpr int F4_LOOK = 2;                       // stages of A scale factors written ahead

template <bool F4>
__global__ void __launch_bounds__(NT, 1) gemm_f8_kernel(const __grid_constant__ Args a) {
  extern __shared__ __align__(1024) uint8_t gsm[];
  uint8_t* base = gsm + ((1024 - (smem_u32(gsm) & 1023)) & 1023);
  const int TT = a.TT;
  const int RB = a.w_bytes + a.a_bytes;  // 16 KB weight tile + TT x 128 B activation tile, both SW128
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + a.RS * RB);
  uint64_t* full = bars;                 // [F8MAXRS] stage landed
  uint64_t* empty = full + F8MAXRS;      // [F8MAXRS] MMAs done with the stage
  uint64_t* accf = empty + F8MAXRS;      // [F8ACC] block accumulator ready
  uint64_t* acce = accf + F8ACC;         // [F8ACC] block accumulator read (one arrival per epilogue warp)
  uint64_t* mdone = acce + F8ACC;        // [1] every MMA of this CTA done
  uint64_t* sfr = mdone + 1;             // [F8MAXRS] FP4: the stage's A scale factors stored (one arrival per quadrant)
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sfr + F8MAXRS);
  volatile int* abortf = reinterpret_cast<volatile int*>(tslot + 1);
  volatile int* lastf = abortf + 1;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x % a.tiles, z = blockIdx.x / a.tiles;
  const int tn = tile % a.tiles_n, tmi = tile / a.tiles_n;
  const int n0 = tn * TM, m0 = tmi * TT;
  const int kb0 = (int)((long long)z * a.nkb / a.S), kb1 = (int)((long long)(z + 1) * a.nkb / a.S);
  const int nk = kb1 - kb0;

  if (tid == 0) {
    for (int s = 0; s < F8MAXRS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < F8ACC; ++s) {
      mbar_init(&accf[s], 1);
      mbar_init(&acce[s], 8);
    }
    mbar_init(mdone, 1);
    for (int s = 0; s < F8MAXRS; ++s) mbar_init(&sfr[s], 4);
    *abortf = 0;
    *lastf = 0;
    fence_mbar_init();
  }
  // FP8: 64, 128, 256 or 512 accumulator columns; FP4 (TT <= 64): accumulators in [0, 256), scale
  // factors from column 320
  const uint32_t ncols = F4 ? 512u : (uint32_t)(F8ACC * TT);
  // accumulators in the ring: four, or two of 128 columns for FP4 at 128 tokens (the scale factors
  // sit from column 320)
  const int nacc = (F4 && TT > 64) ? 2 : F8ACC;
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tslot;
  auto wait = [&](uint64_t* bar, uint32_t par) -> bool {
    if (*abortf) return false;
    if (!mbar_wait(bar, par, kWaitNs)) {
      *abortf = 1;
      return false;
    }
    return true;
  };

  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(&a.tw) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(&a.ta) : "memory");
      int issued = 0;
      for (int i = 0; i < nk; ++i) {
        const int s = i % a.RS;
        if (i >= a.RS && !wait(&empty[s], ((i / a.RS) - 1) & 1)) break;
        uint8_t* st = base + s * RB;
        const int kb = kb0 + i;
        // an FP4 box counts its packed global bytes (the widened shared-memory tile is 16 KB)
        mbar_expect_tx(&full[s], (uint32_t)((F4 ? TM * 64 : a.w_bytes) + a.a_bytes));
        tma_2d(st, &a.tw, kb * 128, n0, &full[s]);
        tma_2d(st + a.w_bytes, &a.ta, kb * 128, m0, &full[s]);
        ++issued;
      }
      for (int i = issued - 1; i >= 0 && i >= issued - a.RS; --i) mbar_wait(&full[i % a.RS], (i / a.RS) & 1, kWaitNs);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = F4 ? (5u << 7) | ((uint32_t)(TT >> 3) << 17) | (1u << 23) | ((uint32_t)(TM >> 4) << 24)
                                : (1u << 4) | ((uint32_t)(TT >> 3) << 17) | ((uint32_t)(TM >> 4) << 24);
      const uint64_t d0 = desc_sw128(smem_u32(base));
      for (int i = 0; i < nk; ++i) {
        const int s = i % a.RS, ac = i % nacc;
        if (!wait(&full[s], (i / a.RS) & 1)) break;
        if (F4 && !wait(&sfr[s], (i / a.RS) & 1)) break;
        if (i >= nacc && !wait(&acce[ac], ((i / nacc) - 1) & 1)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint64_t da = d0 + (uint64_t)((s * RB) >> 4), db = da + (uint64_t)(a.w_bytes >> 4);
        const uint32_t d = tmem + (uint32_t)(ac * TT);
        if (F4) {
          const uint32_t sfa = tmem + F4_SFA + 4u * (uint32_t)s, sfb = tmem + F4_SFB;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            // K step q reads byte q of every scale-factor word
            asm volatile(
                "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d),
                "l"(da + 2u * q), "l"(db + 2u * q), "r"(idesc | ((uint32_t)q << 29) | ((uint32_t)q << 4)),
                "r"(q > 0 ? 1u : 0u), "r"(sfa | ((uint32_t)q << 30)), "r"(sfb | ((uint32_t)q << 30))
                : "memory");
          }
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            asm volatile(
                "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
                "l"(da + 2u * q), "l"(db + 2u * q), "r"(idesc), "r"(q > 0 ? 1u : 0u)
                : "memory");
          }
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                     ::"r"(smem_u32(&empty[s])) : "memory");
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                     ::"r"(smem_u32(&accf[ac])) : "memory");
      }
      // no MMA may still run when the tensor memory is freed
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                   ::"r"(smem_u32(mdone)) : "memory");
      mbar_wait(mdone, 0, kWaitNs);
    }
  } else {
    // ---------------- epilogue: fold each block accumulator with its scales
    const int ct = tid - 64;
    const int qd = warp & 3, half = (warp - 2) >> 2;
    const int row_l = 32 * qd + lane, row = n0 + row_l;
    const int nc = TT / 2, c0 = half * nc;  // 8, 16, 32 or 64 tokens per warp
    const uint32_t tq = tmem + ((uint32_t)(32 * qd) << 16) + (uint32_t)c0;
    const int KS = a.K / 128;
    float acc[64];
#pragma unroll
    for (int c = 0; c < 64; ++c) acc[c] = 0.f;
    // lane l holds the scales (a_s * b_s) of tokens c0 + l and c0 + 32 + l for one block, loaded one
    // block ahead; the folding takes them by shuffle
    auto block_scale = [&](int kb, int h) -> float {
      const int c = 32 * h + lane, t = m0 + c0 + c;
      if (c >= nc || t >= a.M) return 0.f;
      const float bs = F4 ? 1.f : reinterpret_cast<const float*>(a.b_s)[(long long)(n0 / 128) * KS + kb];
      return a.a_s ? a.a_s[(long long)t * KS + kb] * bs : bs;
    };
    // FP4: warps 2-5 (one per lane quadrant) keep the A scale factors in tensor memory. Word c of
    // lane l holds the four 32-K group scales of tile row 32 c + l for one 128-K block; every
    // quadrant holds the same words.
    const bool sf_warp = F4 && half == 0;
    const uint32_t tsf = tmem + ((uint32_t)(32 * qd) << 16);
    auto sf_words = [&](int j, uint32_t (&w)[4]) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int r = n0 + 32 * c + lane;
        w[c] = r < a.N ? *reinterpret_cast<const uint32_t*>(reinterpret_cast<const uint8_t*>(a.b_s) +
                                                            (long long)r * (a.K / 32) + 4 * (kb0 + j))
                       : 0x7F7F7F7Fu;
      }
    };
    auto sf_store = [&](int j, const uint32_t (&w)[4]) -> bool {
      const int s = j % a.RS;
      // the slot's previous stage must be done with its scale factors
      if (j >= a.RS && !wait(&empty[s], ((j / a.RS) - 1) & 1)) return false;
      asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(tsf + F4_SFA + 4u * (uint32_t)s),
                   "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3])
                   : "memory");
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&sfr[s]);
      return true;
    };
    uint32_t swn[4] = {0u, 0u, 0u, 0u};
    if (sf_warp) {
      asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(tsf + F4_SFB),
                   "r"(0x7F7F7F7Fu), "r"(0x7F7F7F7Fu), "r"(0x7F7F7F7Fu), "r"(0x7F7F7F7Fu)
                   : "memory");
      for (int j = 0; j < F4_LOOK && j < nk; ++j) {
        uint32_t w[4];
        sf_words(j, w);
        sf_store(j, w);
      }
      if (F4_LOOK < nk) sf_words(F4_LOOK, swn);
    }
    float sn0 = 0.f, sn1 = 0.f;
    if (nk > 0) {
      sn0 = block_scale(kb0, 0);
      sn1 = block_scale(kb0, 1);
    }
    bool ok = true;
    for (int i = 0; i < nk; ++i) {
      const int ac = i % nacc;
      if (sf_warp && i + F4_LOOK < nk) {
        if (!sf_store(i + F4_LOOK, swn)) {
          ok = false;
          break;
        }
        if (i + F4_LOOK + 1 < nk) sf_words(i + F4_LOOK + 1, swn);
      }
      const float s0 = sn0, s1 = sn1;
      if (i + 1 < nk) {
        sn0 = block_scale(kb0 + i + 1, 0);
        sn1 = block_scale(kb0 + i + 1, 1);
      }
      if (!wait(&accf[ac], (i / nacc) & 1)) {
        ok = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t tb = tq + (uint32_t)(ac * TT);
      if (nc >= 32) {  // 32 or 64 columns: one or two 32-column loads
        {
          float v[32];
          ld32w(tb, v);
#pragma unroll
          for (int q = 0; q < 32; ++q) acc[q] = fmaf(v[q], __shfl_sync(0xffffffffu, s0, q), acc[q]);
        }
        if (nc == 64) {
          float v[32];
          ld32w(tb + 32u, v);
#pragma unroll
          for (int q = 0; q < 32; ++q) acc[32 + q] = fmaf(v[q], __shfl_sync(0xffffffffu, s1, q), acc[32 + q]);
        }
      } else if (nc == 16) {
        float v[16];
        ld16w(tb, v);
#pragma unroll
        for (int q = 0; q < 16; ++q) acc[q] = fmaf(v[q], __shfl_sync(0xffffffffu, s0, q), acc[q]);
      } else {
        float v[8];
        ld8(tb, v);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] = fmaf(v[q], __shfl_sync(0xffffffffu, s0, q), acc[q]);
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[ac]);
    }
    ok = ok && !*abortf;
    const float nanv = __int_as_float(0x7FC00000);
    auto store = [&](int col, float v) {
      const int t = m0 + col;
      if (row < a.N && t < a.M) {
        const long long o = (long long)t * a.N + row;
        if (a.out_f32) reinterpret_cast<float*>(a.out)[o] = v;
        else reinterpret_cast<__nv_bfloat16*>(a.out)[o] = __float2bfloat16_rn(v);
      }
    };
    if (a.S == 1) {
#pragma unroll
      for (int c = 0; c < 64; ++c)
        if (c < nc) store(c0 + c, ok ? acc[c] : nanv);
    } else {
      float* mine = a.part + (long long)blockIdx.x * PART;
#pragma unroll
      for (int c = 0; c < 64; ++c)
        if (c < nc) mine[(c0 + c) * TM + row_l] = ok ? acc[c] : nanv;
      __threadfence();
      named_bar_sync(1, CT);
      if (ct == 0) {
        const unsigned prev = atomicAdd(&a.cnt[tile], 1u);
        *lastf = prev == (unsigned)(a.S - 1);
      }
      named_bar_sync(1, CT);
      if (*lastf) {
        __threadfence();
        for (int c = c0; c < c0 + nc; ++c) {
          float sum = 0.f;
          for (int zz = 0; zz < a.S; ++zz) {
            const float* p = a.part + (long long)(zz * a.tiles + tile) * PART + c * TM + row_l;
            float x;
            asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(x) : "l"(p));
            sum += x;
          }
          store(c, sum);
        }
        if (ct == 0) a.cnt[tile] = 0u;
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
  }
}

// Split-K partial tiles and per-tile arrival counters: static device arrays (10.5 MB, zero at module
// load; the last CTA of a tile resets its counter), so no call allocates.
__device__ float g_split_part[MAXSLOT * PART];
__device__ unsigned g_split_cnt[MAXSLOT];

// ------------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::mutex g_mu;
struct DevState {
  int sms = 0, optin = 0;
  float* part = nullptr;
  unsigned* cnt = nullptr;
  bool attr[2][3] = {{false, false, false}, {false, false, false}};
  bool attr_f8[2] = {false, false};
};
DevState g_dev[64];

int encoder() {
  if (g_encode) return DSMOE_OK;
  cudaDriverEntryPointQueryResult q;
  void* fn = nullptr;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || !fn)
    return cuda_status("gemm: cuTensorMapEncodeTiled entry point");
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return DSMOE_OK;
}

int encode2d(CUtensorMap* m, CUtensorMapDataType dt, const void* p, long long inner, long long rows, long long row_bytes,
             int box0, int box1, CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_NONE) {
  const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  const cuuint32_t box[2] = {(cuuint32_t)box0, (cuuint32_t)box1};
  const cuuint32_t es[2] = {1, 1};
  const CUresult r = g_encode(m, dt, 2, const_cast<void*>(p), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  DSMOE_REQUIRE(r == CUDA_SUCCESS, DSMOE_ERR_CUDA, "gemm: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return DSMOE_OK;
}

template <int FMT, int ADT>
cudaError_t launch(const Args& a, int grid, size_t smem, cudaStream_t st, DevState& d) {
  const int ai = ADT == DSMOE_DTYPE_F32 ? 0 : ADT == DSMOE_DTYPE_BF16 ? 1 : 2;
  if (!d.attr[FMT][ai]) {
    const cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<FMT, ADT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               d.optin);
    if (e != cudaSuccess) return e;
    d.attr[FMT][ai] = true;
  }
  gemm_tc_kernel<FMT, ADT><<<grid, NT, smem, st>>>(a);
  return cudaGetLastError();
}

int launch_gemm(int fmt, const void* x, int a_dtype, const float* a_s, long long M, long long K, const uint8_t* b,
                const void* b_s, long long N, void* out, int out_dtype, void* stream) {
  DSMOE_REQUIRE(x && b && b_s && out, DSMOE_ERR_ARG, "gemm: null pointer");
  DSMOE_REQUIRE(M > 0 && N > 0 && K > 0 && K % 128 == 0, DSMOE_ERR_ARG, "gemm: K (%lld) must be a multiple of 128", K);
  DSMOE_REQUIRE(M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31), DSMOE_ERR_ARG, "gemm: dimension too large");
  DSMOE_REQUIRE(a_dtype == DSMOE_DTYPE_F32 || a_dtype == DSMOE_DTYPE_BF16 || a_dtype == DSMOE_DTYPE_E4M3, DSMOE_ERR_ARG,
                "gemm: a_dtype %d", a_dtype);
  DSMOE_REQUIRE(out_dtype == DSMOE_DTYPE_F32 || out_dtype == DSMOE_DTYPE_BF16, DSMOE_ERR_ARG, "gemm: out_dtype %d",
                out_dtype);
  DSMOE_REQUIRE(((uintptr_t)b & 15) == 0 && ((uintptr_t)x & 15) == 0, DSMOE_ERR_ALIGN,
                "gemm: a and b must be 16-byte aligned");
  DSMOE_REQUIRE(fmt == DSMOE_FMT_FP4 || ((uintptr_t)b_s & 3) == 0, DSMOE_ERR_ALIGN, "gemm: FP8 scales must be 4-byte aligned");
  DSMOE_REQUIRE(a_s == nullptr || ((uintptr_t)a_s & 3) == 0, DSMOE_ERR_ALIGN, "gemm: a_s must be 4-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(g_mu);
  int rc = encoder();
  if (rc) return rc;
  DevState& d = g_dev[dev & 63];
  if (d.sms == 0) {
    cudaDeviceGetAttribute(&d.optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
  }
  Args a{};
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  // e4m3 activations need no conversion: gemm_f8_kernel (FP4 scale words are read 4 bytes at a time)
  const bool f8 = a_dtype == DSMOE_DTYPE_E4M3 && (fmt == DSMOE_FMT_FP8 || ((uintptr_t)b_s & 3) == 0);
  const bool f4n = f8 && fmt == DSMOE_FMT_FP4;
  a.TT = M <= 16 ? 16 : M <= 32 ? 32 : (M <= 192 || !f8) ? TTMAX : F8TTMAX;
  a.tiles_n = (int)((N + TM - 1) / TM);
  const long long tiles = (long long)a.tiles_n * ((M + a.TT - 1) / a.TT);
  DSMOE_REQUIRE(tiles < (1LL << 31), DSMOE_ERR_ARG, "gemm: too many tiles");
  a.tiles = (int)tiles;
  a.nkb = (int)(K / 128);
  // split K over CTAs while the tiles alone leave SMs idle (partials in the static device array)
  int S = 1;
  if (tiles < d.sms) S = (int)std::max<long long>(1, std::min<long long>(std::min<long long>(a.nkb, d.sms / tiles), MAXSLOT / tiles));
  if (S > 1 && !d.part) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(st, &cap);
    if (cap == cudaStreamCaptureStatusNone) {
      // the static partials and counters of this device (nothing is allocated); looked up once
      void* p = nullptr;
      void* c = nullptr;
      if (cudaGetSymbolAddress(&p, g_split_part) != cudaSuccess || cudaGetSymbolAddress(&c, g_split_cnt) != cudaSuccess) {
        cudaGetLastError();
        p = c = nullptr;
      }
      d.part = static_cast<float*>(p);
      d.cnt = static_cast<unsigned*>(c);
      if (!d.part || !d.cnt) d.part = nullptr, d.cnt = nullptr;
    }
  }
  if (!d.part) S = 1;  // first call inside a graph capture: address not looked up yet, no split
  a.S = S;
  a.part = d.part;
  a.cnt = d.cnt;
  const int esz = a_dtype == DSMOE_DTYPE_F32 ? 4 : a_dtype == DSMOE_DTYPE_BF16 ? 2 : 1;
  a.out = out;
  a.out_f32 = out_dtype == DSMOE_DTYPE_F32;
  a.a_s = a_s;
  a.b_s = b_s;
  if (f8) {
    // both operands straight from the TMA into the MMA: FP8 codes x e4m3 codes
    a.w_bytes = TM * 128;
    a.a_bytes = a.TT * 128;
    const size_t rb = (size_t)a.w_bytes + a.a_bytes;
    const int RS = (int)std::min<size_t>(F8MAXRS, ((size_t)d.optin - 1024 - 512) / rb);
    DSMOE_REQUIRE(RS > F4_LOOK, DSMOE_ERR_UNSUPPORTED, "gemm: shared memory for %d stages only", RS);
    a.RS = RS;
    if (f4n)  // packed e2m1: K 4-bit elements per row, K / 2 bytes apart; widened by the TMA
      rc = encode2d(&a.tw, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, b, K, N, K / 2, 128, TM, CU_TENSOR_MAP_SWIZZLE_128B);
    else
      rc = encode2d(&a.tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, b, K, N, K, 128, TM, CU_TENSOR_MAP_SWIZZLE_128B);
    if (!rc) rc = encode2d(&a.ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, x, K, M, K, 128, a.TT, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    const size_t smem = 1024 + (size_t)RS * rb + 512;
    if (!d.attr_f8[f4n]) {
      if (cudaFuncSetAttribute(f4n ? gemm_f8_kernel<true> : gemm_f8_kernel<false>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, d.optin) != cudaSuccess)
        return cuda_status("gemm: set smem");
      d.attr_f8[f4n] = true;
    }
    if (f4n) gemm_f8_kernel<true><<<a.tiles * S, NT, smem, st>>>(a);
    else gemm_f8_kernel<false><<<a.tiles * S, NT, smem, st>>>(a);
    return cuda_status("gemm");
  }
  a.w_bytes = fmt == DSMOE_FMT_FP8 ? TM * 128 : TM * 64;
  a.a_bytes = a.TT * 128 * esz;
  const size_t fixed = 1024 + (size_t)CS * A_BYTES + (size_t)CS * 2 * a.TT * 256 + 256;
  const size_t rb = (size_t)a.w_bytes + a.a_bytes;
  int RS = (int)std::min<size_t>(MAXRS, ((size_t)d.optin - fixed) / rb);
  DSMOE_REQUIRE(RS >= 2, DSMOE_ERR_UNSUPPORTED, "gemm: shared memory for %d raw stages only", RS);
  a.RS = RS;
  const size_t smem = fixed + (size_t)RS * rb;
  // v = a * a_s * b_s is a bf16 value when neither scale applies and a is bf16 or e4m3: no lo term
  a.lo = !(fmt == DSMOE_FMT_FP4 && a_s == nullptr && a_dtype != DSMOE_DTYPE_F32);
  if (fmt == DSMOE_FMT_FP8) rc = encode2d(&a.tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, b, K, N, K, 128, TM);
  else rc = encode2d(&a.tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, b, K / 2, N, K / 2, 64, TM);
  if (rc) return rc;
  const CUtensorMapDataType adt = a_dtype == DSMOE_DTYPE_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                  : a_dtype == DSMOE_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  rc = encode2d(&a.ta, adt, x, K, M, K * esz, 128, a.TT);
  if (rc) return rc;
  const int grid = a.tiles * S;
  cudaError_t e;
  if (fmt == DSMOE_FMT_FP8) {
    e = a_dtype == DSMOE_DTYPE_F32    ? launch<DSMOE_FMT_FP8, DSMOE_DTYPE_F32>(a, grid, smem, st, d)
        : a_dtype == DSMOE_DTYPE_BF16 ? launch<DSMOE_FMT_FP8, DSMOE_DTYPE_BF16>(a, grid, smem, st, d)
                                      : launch<DSMOE_FMT_FP8, DSMOE_DTYPE_E4M3>(a, grid, smem, st, d);
  } else {
    e = a_dtype == DSMOE_DTYPE_F32    ? launch<DSMOE_FMT_FP4, DSMOE_DTYPE_F32>(a, grid, smem, st, d)
        : a_dtype == DSMOE_DTYPE_BF16 ? launch<DSMOE_FMT_FP4, DSMOE_DTYPE_BF16>(a, grid, smem, st, d)
                                      : launch<DSMOE_FMT_FP4, DSMOE_DTYPE_E4M3>(a, grid, smem, st, d);
  }
  if (e != cudaSuccess) {
    set_error("gemm: %s", cudaGetErrorString(e));
    return DSMOE_ERR_CUDA;
  }
  return DSMOE_OK;
}

}  // namespace gemm
}  // namespace dsmoe

using namespace dsmoe;

extern "C" int dsmoe_fp8_gemm(const void* a, int a_dtype, const float* a_s, long long M, long long K, const uint8_t* b,
                              const float* b_s, long long N, void* out, int out_dtype, void* stream) {
  return gemm::launch_gemm(DSMOE_FMT_FP8, a, a_dtype, a_s, M, K, b, b_s, N, out, out_dtype, stream);
}

extern "C" int dsmoe_fp4_gemm(const void* a, int a_dtype, const float* a_s, long long M, long long K, const uint8_t* b,
                              const uint8_t* b_s, long long N, void* out, int out_dtype, void* stream) {
  return gemm::launch_gemm(DSMOE_FMT_FP4, a, a_dtype, a_s, M, K, b, b_s, N, out, out_dtype, stream);
}
