// Prefill / batched MoE layer on the 5th-generation tensor cores (tcgen05, accumulators in TMEM).
//
// Replaces MoE.prefill_batched / _batched (dsv41/tt/moe.py:182-200, 263-288): bincount of the
// (token, expert) pairs, buckets of rows per expert, argsort by expert, gather, batched w1 / w3 /
// w2 matmuls, gather back, routing-weighted sum. Here:
//   group    one CTA sorts the pairs by (expert, token) with a counting sort (deterministic) and cuts
//            each expert's tokens into chunks of <= 64; the shared expert takes every token.
//   tokens   per-token power-of-two prescale, then each chunk's token rows as e4m3 hi / lo pairs
//            (x ~ hi + lo / 16), gathered into the K-major 128-byte-swizzled layout tcgen05 reads.
//   gemm 1   grouped w1|w3: D[128 weight rows][2 n tokens] per (chunk, 64-row M tile), K = hidden.
//   swiglu   h = SiLU(min(g, 10)) * clamp(u, +-10), stored like the tokens (h x 4 in e4m3 hi / lo).
//   gemm 2   grouped w2: D[128 output rows][2 n], K = the intermediate slice.
//   combine  y[t] = sum_k wt[t][k] * y_pair[t, k] + y_shared[t], in k order (deterministic).
// GEMM kernel: one CTA per SM walks (chunk, M tile) units. Warp 0 lane 0 streams each 128-K step's
// packed weight pieces and the chunk's token rows with 1-D bulk copies; warps 2-9 rearrange the
// packed weights (the decode store's lane-fragment order) into the canonical K-major SW128 tile,
// expanding FP4 to e4m3; warp 1 lane 0 issues tcgen05.mma (M 128, N = 2 x tokens, K 32 per
// instruction) with the accumulator in TMEM; warps 2-9 read it back with tcgen05.ld (two warps per
// TMEM lane quadrant, splitting the columns).
//   FP8 weights (fp32 scale per 128 x 128 block): kind::f8f6f4, one TMEM block accumulator per
//     128-K step (two, alternating); the epilogue warps fold each block into a TMEM running sum
//     with the block's scale (the non-MX scales applied per K block to the accumulator).
//   FP4 weights (e8m0 per 32): kind::mxf8f6f4.block_scale with the e4m3-expanded weights, the
//     checkpoint's e8m0 scales (+6, undoing the expansion's 2^-6) as the A scale factors in TMEM
//     and 1.0 for B: the tensor core applies the block scales itself.
// Every wait is bounded; an expired wait sets a status bit (checked by dsmoe_moe_check).
#include "router.cuh"

namespace dsmoe {

constexpr int PFW = 10, PFT = PFW * 32;  // warps: 0 producer, 1 MMA, 2-9 convert + epilogue
constexpr int PCW = PFW - 2, PCT = PCW * 32;  // convert + epilogue warps / threads (two per TMEM lane quadrant)
constexpr int PST = 4;                   // pipeline stages (128-K steps)
constexpr int PCHUNK = 64;               // tokens per chunk
constexpr int PNMAX = 2 * PCHUNK;        // MMA N: hi and lo rows of every token
constexpr int PA_BYTES = 16384;          // A tile: 128 rows x 128 K e4m3, SW128
constexpr int PB_BYTES = PNMAX * 128;    // B tile: up to 128 rows x 128 K
constexpr int PRAW_BYTES = 16896;        // packed weight pieces of one step (<= 16416 used)
constexpr int PSTAGE = PA_BYTES + PB_BYTES + PRAW_BYTES;
constexpr int PSMEM = PST * PSTAGE + 2048;  // + 1024-byte alignment slack, barriers, flags
constexpr uint64_t kPWaitNs = 1000000000ull;
// TMEM columns: FP8 block accumulators 0 / 128, running sum 256; FP4 accumulator 0; A scale
// factors 384 + 4 * stage; B scale factors 400.
constexpr uint32_t TM_RUN = 256, TM_SFA = 384, TM_SFB = 400;

enum : unsigned { PST_WAIT = 32u, PST_ROUTE = 64u };

struct PChunk {
  int expert;  // routed expert, or -1 for the shared expert
  int pair0;   // first pair (sorted order) of the chunk
  int n;       // tokens
  int npad;    // n rounded up to 8: the MMA N is 2 * npad
  long long bofs;  // rows (of 128 B) before the chunk's block in the B buffer; the block of a GEMM with
                   // K = 128 * katoms starts at byte bofs * katoms * 128 and is [katoms][2 npad][128 B]
};

struct GroupOut {
  int* cnt;         // [E]
  int* pair_tok;    // [P * (k + 1)]: token of each pair, sorted by (expert, token); shared pairs last
  int* pos_of;      // [P * k]: sorted position of pair (t, k)
  PChunk* chunks;   // [max chunks]
  int* nchunks;     // [1]
  long long* bytes; // [1]: B-buffer rows (sum over chunks of 2 npad)
};

__host__ __device__ inline int prefill_max_chunks(int P, int topk, int E) {
  return E + (P * topk + PCHUNK - 1) / PCHUNK + (P + PCHUNK - 1) / PCHUNK;
}

// ------------------------------------------------------------------ grouping (one CTA)
__global__ void __launch_bounds__(1024) prefill_group_kernel(const int64_t* idx, int P, int topk, int E,
                                                             GroupOut g, unsigned* status) {
  extern __shared__ int gsm[];
  int* cnt = gsm;            // [E]
  int* off = cnt + E;        // [E + 1]
  short* ids = reinterpret_cast<short*>(off + E + 1);  // [P * topk]
  const int tid = threadIdx.x, np = P * topk;
  for (int e = tid; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int i = tid; i < np; i += blockDim.x) {
    long long e = idx[i];
    if (e < 0 || e >= E) {
      atomicOr(status, PST_ROUTE);
      e = 0;
    }
    ids[i] = (short)e;
    atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  if (tid == 0) {
    int s = 0;
    for (int e = 0; e < E; ++e) {
      off[e] = s;
      s += cnt[e];
    }
    off[E] = s;
  }
  __syncthreads();
  // expert e's pairs in token order: thread e walks the tokens (a token picks an expert once)
  for (int e = tid; e < E; e += blockDim.x) {
    g.cnt[e] = cnt[e];
    if (cnt[e] == 0) continue;
    int pos = off[e];
    for (int i = 0; i < np; ++i)
      if (ids[i] == e) {
        g.pair_tok[pos] = i / topk;
        g.pos_of[i] = pos;
        ++pos;
      }
  }
  for (int t = tid; t < P; t += blockDim.x) g.pair_tok[np + t] = t;
  __syncthreads();
  if (tid == 0) {  // chunks: each expert's pairs in runs of <= PCHUNK, then the shared expert's
    int nc = 0;
    long long bo = 0;
    auto add = [&](int e, int p0, int n) {
      PChunk c;
      c.expert = e;
      c.pair0 = p0;
      c.n = n;
      c.npad = (n + 7) & ~7;
      c.bofs = bo;
      bo += 2LL * c.npad;
      g.chunks[nc++] = c;
    };
    for (int e = 0; e < E; ++e)
      for (int c0 = 0; c0 < cnt[e]; c0 += PCHUNK) add(e, off[e] + c0, min(PCHUNK, cnt[e] - c0));
    for (int c0 = 0; c0 < P; c0 += PCHUNK) add(-1, np + c0, min(PCHUNK, P - c0));
    *g.nchunks = nc;
    *g.bytes = bo;
  }
}

// Per-token power-of-two prescale: x * 2^-p has its largest magnitude in [128, 256).
__global__ void prefill_token_scale_kernel(const __nv_bfloat16* x, int P, int H, float* xscale) {
  const int t = blockIdx.x;
  if (t >= P) return;
  float m = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) m = fmaxf(m, fabsf(__bfloat162float(x[(long long)t * H + i])));
  m = warp_max(m);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float mm = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) mm = fmaxf(mm, red[w]);
    int p = 0;
    if (mm > 0.f && mm <= 3.0e38f) {
      int e2;
      frexpf(mm, &e2);
      p = e2 - 8;
    }
    xscale[t] = ldexpf(1.0f, p);
  }
}

// Offset of 16-byte chunk cc (0..7) of row r in a K-major SW128 tile with 128-byte rows.
__host__ __device__ __forceinline__ uint32_t sw128(int r, int cc) { return (uint32_t)(r * 128 + ((cc ^ (r & 7)) << 4)); }

// B operand rows of every chunk: [K / 128][2 npad rows][128 B] per chunk, row j < npad the hi
// part of token j, row npad + j its lo part (zero rows past n). One thread per 16 bytes.
// src(pair, k) is x[tok] * 2^-p (phase 1) or h (phase 2); both come through `value`.
template <class V>
__device__ __forceinline__ void write_b_rows(const PChunk& c, int K, int item, uint8_t* dst, V&& value) {
  const int ka = item / (2 * c.npad * 8), rem = item - ka * 2 * c.npad * 8;
  const int r = rem >> 3, cc = rem & 7;
  const int j = r < c.npad ? r : r - c.npad;
  const bool lo = r >= c.npad;
  uint32_t w[4] = {0u, 0u, 0u, 0u};
  if (j < c.n) {
    float v[16];
    value(c.pair0 + j, ka * 128 + cc * 16, v);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      uint32_t hi2, lo2;
      split2_e4m3(v[2 * q], v[2 * q + 1], hi2, lo2);
      const uint32_t b2 = lo ? lo2 : hi2;
      w[q >> 1] |= b2 << (16 * (q & 1));
    }
  }
  *reinterpret_cast<uint4*>(dst + c.bofs * K + (long long)ka * 2 * c.npad * 128 + sw128(r, cc)) =
      make_uint4(w[0], w[1], w[2], w[3]);
}

struct TokArgs {
  const __nv_bfloat16* x;
  int H, I_loc;
  const PChunk* chunks;
  const int* nchunks;
  const int* pair_tok;
  const float* xscale;
  const float* gu;  // phase 2: [pairs][2 I_loc] g | u
  uint8_t* dst;
};

// One CTA per chunk (grid = max chunks); phase 1 = tokens, phase 2 = SwiGLU of gemm 1's output.
template <int PH>
__global__ void prefill_rows_kernel(TokArgs a) {
  const int ci = blockIdx.x;
  if (ci >= *a.nchunks) return;
  const PChunk c = a.chunks[ci];
  const int K = PH == 1 ? a.H : a.I_loc;
  const int items = (K / 128) * 2 * c.npad * 8;
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    if (PH == 1) {
      write_b_rows(c, K, it, a.dst, [&](int pair, int k0, float* v) {
        const int tok = a.pair_tok[pair];
        const float inv = 1.0f / a.xscale[tok];
        const uint4* src = reinterpret_cast<const uint4*>(a.x + (long long)tok * a.H + k0);
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const uint4 u = src[q];
          const uint32_t ww[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            v[8 * q + 2 * h] = __uint_as_float(ww[h] << 16) * inv;
            v[8 * q + 2 * h + 1] = __uint_as_float(ww[h] & 0xFFFF0000u) * inv;
          }
        }
      });
    } else {
      write_b_rows(c, K, it, a.dst, [&](int pair, int k0, float* v) {
        const float* gp = a.gu + (long long)pair * 2 * a.I_loc + k0;
        const float* up = gp + a.I_loc;
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const float gv = fminf(gp[q], 10.0f);
          const float uv = fminf(fmaxf(up[q], -10.0f), 10.0f);
          v[q] = gv / (1.0f + expf(-gv)) * uv * kHScale;
        }
      });
    }
  }
}

// ------------------------------------------------------------------ tcgen05 helpers
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_mma_f8(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void tc_mma_mx(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t sfa,
                                          uint32_t sfb, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb)
      : "memory");
}
__device__ __forceinline__ void tc_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tc_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
      : "memory");
}
__device__ __forceinline__ void tc_st4(uint32_t taddr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ------------------------------------------------------------------ the grouped GEMM
struct GemmArgs {
  int phase;  // 1: w1|w3 -> gu, 2: w2 -> y_pair
  int H, I_loc, r_fmt;
  const uint8_t* r_base;  // routed store of this phase
  long long r_eb;         // bytes per routed expert
  long long tile_r;       // bytes per 16-row tile (routed format)
  const uint8_t* s_base;  // shared expert (FP8) store of this phase
  long long tile_s;
  int KC_r8, KC_s;        // FP8 chunk counts per tile row (scale offsets)
  const PChunk* chunks;
  const int* nchunks;
  const uint8_t* bsrc;
  int katoms, mtiles;
  float* out;
  int out_ld;
  const int* pair_tok;
  const float* xscale;  // phase 1: per token; phase 2: unused
  unsigned* status;
};

struct PUnit {
  const uint8_t* tile0;  // first packed 16-row tile of the M tile
  long long tile;        // bytes per tile
  int fmt, KC;
  PChunk c;
  int mt;
};

__device__ __forceinline__ PUnit punit(const GemmArgs& a, int u) {
  PUnit p;
  const int ci = u / a.mtiles;
  p.mt = u - ci * a.mtiles;
  p.c = a.chunks[ci];
  const bool sh = p.c.expert < 0;
  p.fmt = sh ? DSMOE_FMT_FP8 : a.r_fmt;
  p.tile = sh ? a.tile_s : a.tile_r;
  p.KC = sh ? a.KC_s : a.KC_r8;
  const uint8_t* base = sh ? a.s_base : a.r_base + (long long)p.c.expert * a.r_eb;
  p.tile0 = base + (long long)(a.phase == 1 ? 4 : 8) * p.mt * p.tile;
  return p;
}

__global__ void __launch_bounds__(PFT, 1) prefill_gemm_kernel(GemmArgs a) {
  extern __shared__ __align__(1024) uint8_t psm[];
  uint8_t* base = psm + ((1024 - (smem_u32(psm) & 1023)) & 1023);  // 1024-aligned (SW128 atoms)
  uint8_t* sA = base;                        // [PST][PA_BYTES]
  uint8_t* sB = sA + PST * PA_BYTES;         // [PST][PB_BYTES]
  uint8_t* sR = sB + PST * PB_BYTES;         // [PST][PRAW_BYTES]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sR + PST * PRAW_BYTES);
  uint64_t* full = bars;            // [PST] producer's copies landed
  uint64_t* afull = full + PST;     // [PST] A tile converted (one arrival per converting warp)
  uint64_t* sfree = afull + PST;    // [PST] MMAs done with the stage
  uint64_t* bdone = sfree + PST;    // [2] FP8 block accumulator ready
  uint64_t* bfree = bdone + 2;      // [2] FP8 block accumulator folded (one arrival per epilogue warp)
  uint64_t* udone = bfree + 2;      // [1] FP4 unit accumulator ready
  uint64_t* ufree = udone + 1;      // [1] unit result read (one arrival per epilogue warp)
  uint64_t* endb = ufree + 1;       // [1] every MMA of this CTA done
  uint64_t* efin = endb + 1;        // [1] FP8 running sum complete (one arrival per epilogue warp)
  uint32_t* tslot = reinterpret_cast<uint32_t*>(efin + 1);
  volatile int* abortf = reinterpret_cast<volatile int*>(tslot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nunits = *a.nchunks * a.mtiles;
  const int G = gridDim.x;
  if (tid == 0) {
    for (int s = 0; s < PST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&afull[s], PCW);
      mbar_init(&sfree[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bdone[b], 1);
      mbar_init(&bfree[b], PCW);
    }
    mbar_init(udone, 1);
    mbar_init(ufree, PCW);
    mbar_init(endb, 1);
    mbar_init(efin, PCW);
    *abortf = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)), "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = *tslot;
  auto fail = [&](unsigned bit) {
    atomicOr(a.status, bit);
    *abortf = 1;
  };
  auto wait = [&](uint64_t* bar, uint32_t par) -> bool {
    if (*abortf) return false;
    if (!mbar_wait(bar, par, kPWaitNs)) {
      fail(PST_WAIT);
      return false;
    }
    return true;
  };

  if (warp == 0) {
    // ---------------- producer
    if (lane == 0) {
      const uint64_t pol = l2_evict_first();
      int it = 0;
      for (int u = blockIdx.x; u < nunits && !*abortf; u += G) {
        const PUnit p = punit(a, u);
        const int nb = 2 * p.c.npad * 128;
        for (int ka = 0; ka < a.katoms; ++ka, ++it) {
          const int s = it % PST;
          if (it >= PST && !wait(&sfree[s], ((it / PST) - 1) & 1)) break;
          uint8_t* raw = sR + s * PRAW_BYTES;
          uint32_t bytes = (uint32_t)nb;
          if (p.fmt == DSMOE_FMT_FP8) bytes += a.phase == 1 ? 4 * 4096 + 16 : 8 * 2048 + 32;
          else bytes += a.phase == 1 ? 4 * 2176 : 8 * 1088;
          mbar_expect_tx(&full[s], bytes);
          const uint8_t* bsrc = a.bsrc + p.c.bofs * 128 * a.katoms + (long long)ka * nb;
          bulk_g2s(sB + s * PB_BYTES, bsrc, (uint32_t)nb, &full[s]);
          if (p.fmt == DSMOE_FMT_FP8) {
            if (a.phase == 1) {
              for (int tt = 0; tt < 4; ++tt)
                bulk_g2s_hint(raw + tt * 4096, p.tile0 + tt * p.tile + (long long)(ka >> 1) * kFp8W13Item + (ka & 1) * 4096,
                              4096, &full[s], pol);
              bulk_g2s_hint(raw + 16384, p.tile0 + fp8_w13_scale_off(ka >> 1, p.KC), 16, &full[s], pol);
            } else {
              for (int tt = 0; tt < 8; ++tt)
                bulk_g2s_hint(raw + tt * 2048, p.tile0 + tt * p.tile + (long long)(ka >> 1) * kFp8W2Item + (ka & 1) * 2048,
                              2048, &full[s], pol);
              bulk_g2s_hint(raw + 16384, p.tile0 + fp8_w2_scale_off(ka >> 1, p.KC), 32, &full[s], pol);
            }
          } else {
            if (a.phase == 1) {
              for (int tt = 0; tt < 4; ++tt)
                bulk_g2s_hint(raw + tt * 2176, p.tile0 + tt * p.tile + (long long)ka * 2176, 2176, &full[s], pol);
            } else {
              for (int tt = 0; tt < 8; ++tt)
                bulk_g2s_hint(raw + tt * 1088, p.tile0 + tt * p.tile + (long long)ka * 1088, 1088, &full[s], pol);
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      int it = 0, nblk = 0, nmx = 0, nu = 0;
      for (int u = blockIdx.x; u < nunits && !*abortf; u += G, ++nu) {
        const PUnit p = punit(a, u);
        const int N = 2 * p.c.npad;
        const bool mx = p.fmt == DSMOE_FMT_FP4;
        if (nu > 0 && !wait(ufree, (nu - 1) & 1)) break;
        tc_fence_after();
        const uint32_t idesc8 = (1u << 4) | ((uint32_t)(N >> 3) << 17) | (8u << 24);
        const uint32_t idescx = ((uint32_t)(N >> 3) << 17) | (1u << 23) | (8u << 24);
        bool ok = true;
        for (int ka = 0; ka < a.katoms; ++ka, ++it) {
          const int s = it % PST;
          if (!wait(&afull[s], (it / PST) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t abase = smem_u32(sA + s * PA_BYTES), bbase = smem_u32(sB + s * PB_BYTES);
          if (!mx) {
            const int bb = nblk & 1;
            if (nblk >= 2 && !wait(&bfree[bb], ((nblk >> 1) - 1) & 1)) {
              ok = false;
              break;
            }
            tc_fence_after();
            for (int k = 0; k < 4; ++k)
              tc_mma_f8(tm + 128u * bb, umma_desc_sw128(abase + 32 * k), umma_desc_sw128(bbase + 32 * k), idesc8,
                        k > 0 ? 1u : 0u);
            tc_commit(&sfree[s]);
            tc_commit(&bdone[bb]);
            ++nblk;
          } else {
            for (int k = 0; k < 4; ++k) {
              const uint32_t id = idescx | ((uint32_t)k << 29) | ((uint32_t)k << 4);
              tc_mma_mx(tm, umma_desc_sw128(abase + 32 * k), umma_desc_sw128(bbase + 32 * k), id,
                        (tm + TM_SFA + 4 * s) | ((uint32_t)k << 30), (tm + TM_SFB) | ((uint32_t)k << 30),
                        (ka > 0 || k > 0) ? 1u : 0u);
            }
            tc_commit(&sfree[s]);
          }
        }
        if (!ok) break;
        if (mx) {
          tc_commit(udone);
          ++nmx;
        }
      }
      (void)nmx;
      tc_commit(endb);  // completes once every MMA issued above has
      mbar_wait(endb, 0, kPWaitNs);
    }
  } else {
    // ---------------- convert + epilogue (warps 2-9: TMEM lane quadrant q = warp % 4, column half hf)
    const int q = warp & 3, c = tid - 64, hf = (warp - 2) >> 2;
    const uint32_t trow = tm + ((uint32_t)(32 * q) << 16);
    if (hf == 0) {
      tc_st4(trow + TM_SFB, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu);  // B scale factors: 1.0
      tc_wait_st();
    }
    const int R = 32 * q + lane;  // this thread's accumulator row
    int it = 0, nblk = 0, nmx = 0, nfin = 0;
    float pend_scale = 0.f;
    // fold FP8 block accumulator (the step before) into the running sum with its scale
    auto epi_block = [&](int kb, float sc, int N) -> bool {
      const int bb = nblk & 1;
      if (!wait(&bdone[bb], (nblk >> 1) & 1)) return false;
      tc_fence_after();
      for (int c0 = 16 * hf; c0 < N; c0 += 32) {
        float blk[16], run[16];
        tc_ld16(trow + 128u * bb + c0, blk);
        if (kb > 0) tc_ld16(trow + TM_RUN + c0, run);
        tc_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) run[i] = kb > 0 ? fmaf(blk[i], sc, run[i]) : blk[i] * sc;
        tc_st16(trow + TM_RUN + c0, run);
      }
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bfree[bb]);
      ++nblk;
      return true;
    };
    for (int u = blockIdx.x; u < nunits && !*abortf; u += G) {
      const PUnit p = punit(a, u);
      const int N = 2 * p.c.npad;
      const bool mx = p.fmt == DSMOE_FMT_FP4;
      bool ok = true;
      for (int ka = 0; ka < a.katoms; ++ka, ++it) {
        const int s = it % PST;
        if (!wait(&full[s], (it / PST) & 1)) {
          ok = false;
          break;
        }
        const uint8_t* raw = sR + s * PRAW_BYTES;
        uint8_t* At = sA + s * PA_BYTES;
        float sc = 0.f;
        if (!mx) {
          // FP8 lane fragments -> K-major SW128 rows (4-byte pieces)
          const int nfr = 1024;
          for (int f = c; f < nfr; f += PCT) {
            int l, R0, ch;
            const uint8_t* src;
            if (a.phase == 1) {
              l = f & 31;
              const int m = (f >> 5) & 1;
              ch = (f >> 6) & 3;
              const int tt = f >> 8;
              src = raw + tt * 4096 + ch * 1024 + m * 512 + l * 16;
              R0 = m * 64 + 16 * tt;
            } else {
              l = f & 31;
              ch = (f >> 5) & 3;
              const int tt = f >> 7;
              src = raw + tt * 2048 + ch * 512 + l * 16;
              R0 = 16 * tt;
            }
            const uint4 v = *reinterpret_cast<const uint4*>(src);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
            const int g = l >> 2, t = l & 3;
#pragma unroll
            for (int r = 0; r < 4; ++r) {
              const int row = R0 + g + 8 * (r & 1), kk = 32 * ch + 4 * t + 16 * (r >> 1);
              *reinterpret_cast<uint32_t*>(At + sw128(row, kk >> 4) + (kk & 15)) = w[r];
            }
          }
          const float* sp = reinterpret_cast<const float*>(raw + 16384);
          if (a.phase == 1)
            sc = sp[fp8_w13_scale_index(ka, R >= 64 ? 1 : 0)];
          else
            sc = sp[(4 * ka) & 7];
        } else {
          // FP4 lane fragments -> e4m3 (x 2^-6) in K-major SW128 rows; e8m0 scales (+6) -> TMEM
          const int nfr = 512;
          for (int f = c; f < nfr; f += PCT) {
            int l, R0, ch;
            const uint8_t* src;
            if (a.phase == 1) {
              l = f & 31;
              const int m = (f >> 5) & 1;
              ch = (f >> 6) & 1;
              const int tt = f >> 7;
              src = raw + tt * 2176 + ch * 1088 + m * 512 + l * 16;
              R0 = m * 64 + 16 * tt;
            } else {
              l = f & 31;
              ch = (f >> 5) & 1;
              const int tt = f >> 6;
              src = raw + tt * 1088 + ch * 544 + l * 16;
              R0 = 16 * tt;
            }
            const uint4 v = *reinterpret_cast<const uint4*>(src);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
            const int g = l >> 2, t = l & 3;
#pragma unroll
            for (int ww = 0; ww < 4; ++ww) {
              uint32_t lo, hi;
              fp4w_to_e4m3(w[ww], lo, hi);
              const int row = R0 + g + 8 * (ww & 1), kk = 64 * ch + 32 * (ww >> 1) + 4 * t;
              *reinterpret_cast<uint32_t*>(At + sw128(row, kk >> 4) + (kk & 15)) = lo;
              *reinterpret_cast<uint32_t*>(At + sw128(row, (kk + 16) >> 4) + ((kk + 16) & 15)) = hi;
            }
          }
          if (hf == 0) {
          uint32_t sf[4];
#pragma unroll
          for (int m1 = 0; m1 < 4; ++m1) {
            const int Rr = lane + 32 * m1;
            uint32_t word = 0;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
              const int ch = b >> 1, gp = b & 1;
              int off;
              if (a.phase == 1) {
                const int m = Rr >= 64 ? 1 : 0, tt = (Rr & 63) >> 4, rr = Rr & 15;
                off = tt * 2176 + ch * 1088 + 1024 + m * 32 + 4 * (rr & 7) + 2 * (rr >> 3) + gp;
              } else {
                const int tt = Rr >> 4, rr = Rr & 15;
                off = tt * 1088 + ch * 544 + 512 + 4 * (rr & 7) + 2 * (rr >> 3) + gp;
              }
              uint32_t e = raw[off];
              if (e != 0xFFu) e = min(e + 6u, 254u);
              word |= e << (8 * b);
            }
            sf[m1] = word;
          }
          tc_st4(trow + TM_SFA + 4 * s, sf[0], sf[1], sf[2], sf[3]);
          tc_wait_st();
          }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&afull[s]);
        if (!mx) {
          if (ka > 0 && !epi_block(ka - 1, pend_scale, N)) {
            ok = false;
            break;
          }
          pend_scale = sc;
        }
      }
      if (!ok) break;
      uint32_t src_col;
      if (!mx) {
        if (!epi_block(a.katoms - 1, pend_scale, N)) break;
        // the two warps of a quadrant wrote alternate 16-column chunks of the running sum; the hi /
        // lo columns of a token can sit in chunks of different warps, so all folds finish first
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(efin);
        if (!wait(efin, nfin & 1)) break;
        ++nfin;
        tc_fence_after();
        src_col = TM_RUN;
      } else {
        if (!wait(udone, nmx & 1)) break;
        tc_fence_after();
        ++nmx;
        src_col = 0;
      }
      // unit result: row R, columns j (hi) and npad + j (lo) of token j
      // (16-column loads may read up to 8 columns past N; those values belong to no token)
      const int npad = p.c.npad;
      for (int j0 = 16 * hf; j0 < npad; j0 += 32) {
        float hv[16], lv[16];
        tc_ld16(trow + src_col + j0, hv);
        tc_ld16(trow + src_col + npad + j0, lv);
        tc_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int j = j0 + i;
          if (j >= p.c.n) break;
          float v = hv[i] + lv[i] * (1.0f / kLoScale);
          const int pair = p.c.pair0 + j;
          long long col;
          if (a.phase == 1) {
            v *= a.xscale[a.pair_tok[pair]];
            col = (R >= 64 ? a.I_loc : 0) + 64 * p.mt + (R & 63);
          } else {
            v *= 1.0f / kHScale;
            col = 128LL * p.mt + R;
          }
          a.out[(long long)pair * a.out_ld + col] = v;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(ufree);
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tm), "r"(512) : "memory");
  }
}

// y[t] = sum_k wt[t][k] * y_pair[pos(t, k)] + y_pair[shared t], k in order.
__global__ void prefill_combine_kernel(const float* ypair, const int* pos_of, const float* wt, int P, int topk,
                                       int H, void* y, int y_f32) {
  const int t = blockIdx.y;
  for (int h = blockIdx.x * blockDim.x + threadIdx.x; h < H; h += gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < topk; ++k) s += wt[t * topk + k] * ypair[(long long)pos_of[t * topk + k] * H + h];
    s += ypair[(long long)(P * topk + t) * H + h];
    if (y_f32)
      reinterpret_cast<float*>(y)[(long long)t * H + h] = s;
    else
      reinterpret_cast<__nv_bfloat16*>(y)[(long long)t * H + h] = __float2bfloat16_rn(s);
  }
}

// ------------------------------------------------------------------ host side
struct PrefillWs {
  size_t status, cnt, pair_tok, pos_of, chunks, nchunks, bytes, xscale, bbuf1, bbuf2, gu, ypair, idx, wt, logits,
      rscr, total;
  long long bbuf1_bytes, bbuf2_bytes;
};

static size_t pal(size_t v) { return (v + 255) & ~size_t(255); }

PrefillWs prefill_ws(int P, int H, int I_loc, int E, int topk) {
  PrefillWs w{};
  const long long np = (long long)P * topk, npa = np + P;
  const int maxc = prefill_max_chunks(P, topk, E);
  const long long rows = npa + 8LL * maxc;  // sum over chunks of npad
  size_t o = 0;
  w.status = o; o += pal(4);
  w.cnt = o; o += pal((size_t)E * 4);
  w.pair_tok = o; o += pal((size_t)npa * 4);
  w.pos_of = o; o += pal((size_t)np * 4);
  w.chunks = o; o += pal((size_t)maxc * sizeof(PChunk));
  w.nchunks = o; o += pal(4);
  w.bytes = o; o += pal(8);
  w.xscale = o; o += pal((size_t)P * 4);
  w.bbuf1_bytes = 2 * rows * H;
  w.bbuf2_bytes = 2 * rows * I_loc;
  w.bbuf1 = o; o += pal((size_t)w.bbuf1_bytes);
  w.bbuf2 = o; o += pal((size_t)w.bbuf2_bytes);
  w.gu = o; o += pal((size_t)npa * 2 * I_loc * 4);
  w.ypair = o; o += pal((size_t)npa * H * 4);
  w.idx = o; o += pal((size_t)np * 8);
  w.wt = o; o += pal((size_t)np * 4);
  w.total = o;
  return w;
}

}  // namespace dsmoe

using namespace dsmoe;

static int prefill_validate(const dsmoe_layer_t* L, int P) {
  DSMOE_REQUIRE(L, DSMOE_ERR_ARG, "prefill: layer is null");
  DSMOE_REQUIRE(P >= 1 && P <= 4096, DSMOE_ERR_ARG, "prefill: tokens %d outside 1..4096", P);
  DSMOE_REQUIRE(L->hidden > 0 && L->hidden % 128 == 0, DSMOE_ERR_ARG, "prefill: hidden %d must be a multiple of 128",
                L->hidden);
  DSMOE_REQUIRE(L->inter_local > 0 && L->inter_local % 128 == 0, DSMOE_ERR_UNSUPPORTED,
                "prefill: inter_local %d must be a multiple of 128", L->inter_local);
  DSMOE_REQUIRE(L->n_experts >= 1 && L->n_experts <= 4096 && L->topk >= 1 && L->topk <= DSMOE_MAX_TOPK, DSMOE_ERR_ARG,
                "prefill: n_experts %d / topk %d", L->n_experts, L->topk);
  DSMOE_REQUIRE((long long)P * L->topk <= 8192, DSMOE_ERR_ARG, "prefill: %d pairs > 8192", P * L->topk);
  DSMOE_REQUIRE(L->routed.fmt == DSMOE_FMT_FP8 || L->routed.fmt == DSMOE_FMT_FP4, DSMOE_ERR_ARG, "prefill: fmt %d",
                L->routed.fmt);
  DSMOE_REQUIRE(L->shared.fmt == DSMOE_FMT_FP8 && L->shared.n_experts == 1, DSMOE_ERR_UNSUPPORTED,
                "prefill: the shared expert must be one FP8 expert");
  DSMOE_REQUIRE(L->routed.w13 && L->routed.w2 && L->shared.w13 && L->shared.w2, DSMOE_ERR_ARG,
                "prefill: expert stores are null");
  return DSMOE_OK;
}

extern "C" size_t dsmoe_moe_prefill_workspace_bytes(const dsmoe_layer_t* L, int P) {
  if (prefill_validate(L, P) != DSMOE_OK) return 0;
  return prefill_ws(P, L->hidden, L->inter_local, L->n_experts, L->topk).total;
}

extern "C" int dsmoe_moe_prefill(const dsmoe_layer_t* L, const void* x, int P, const int64_t* idx, const float* wt,
                                 void* y, int y_dtype, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = prefill_validate(L, P);
  if (rc) return rc;
  DSMOE_REQUIRE(x && idx && wt && y && workspace, DSMOE_ERR_ARG, "prefill: x / idx / wt / y / workspace null");
  DSMOE_REQUIRE(y_dtype == DSMOE_DTYPE_BF16 || y_dtype == DSMOE_DTYPE_F32, DSMOE_ERR_ARG, "prefill: y_dtype %d", y_dtype);
  DSMOE_REQUIRE(((uintptr_t)x & 15) == 0 && ((uintptr_t)workspace & 255) == 0, DSMOE_ERR_ALIGN,
                "prefill: x must be 16-byte and workspace 256-byte aligned");
  const int H = L->hidden, I = L->inter_local, E = L->n_experts, K = L->topk;
  const PrefillWs w = prefill_ws(P, H, I, E, K);
  DSMOE_REQUIRE(workspace_bytes >= w.total, DSMOE_ERR_WORKSPACE, "prefill: workspace %zu < %zu", workspace_bytes, w.total);
  cudaStream_t st = (cudaStream_t)stream;
  uint8_t* ws = (uint8_t*)workspace;
  unsigned* status = (unsigned*)(ws + w.status);
  const int maxc = prefill_max_chunks(P, K, E);

  GroupOut g{(int*)(ws + w.cnt), (int*)(ws + w.pair_tok), (int*)(ws + w.pos_of), (PChunk*)(ws + w.chunks),
             (int*)(ws + w.nchunks), (long long*)(ws + w.bytes)};
  const size_t gsm = (size_t)(2 * E + 1) * 4 + (size_t)P * K * 2;
  if (gsm > 48 * 1024) cudaFuncSetAttribute(prefill_group_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gsm);
  prefill_group_kernel<<<1, 1024, gsm, st>>>(idx, P, K, E, g, status);
  prefill_token_scale_kernel<<<P, 256, 0, st>>>((const __nv_bfloat16*)x, P, H, (float*)(ws + w.xscale));

  TokArgs ta{};
  ta.x = (const __nv_bfloat16*)x;
  ta.H = H;
  ta.I_loc = I;
  ta.chunks = g.chunks;
  ta.nchunks = g.nchunks;
  ta.pair_tok = g.pair_tok;
  ta.xscale = (const float*)(ws + w.xscale);
  ta.gu = (const float*)(ws + w.gu);
  ta.dst = ws + w.bbuf1;
  prefill_rows_kernel<1><<<maxc, 256, 0, st>>>(ta);

  static int attr_set[64], sm_count[64];  // per device, set once
  int dev = 0;
  cudaGetDevice(&dev);
  dev &= 63;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(prefill_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PSMEM) != cudaSuccess)
      return cuda_status("prefill: gemm smem");
    cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
    attr_set[dev] = 1;
  }
  const int sms = sm_count[dev];

  GemmArgs ga{};
  ga.phase = 1;
  ga.H = H;
  ga.I_loc = I;
  ga.r_fmt = L->routed.fmt;
  ga.r_base = L->routed.w13;
  ga.r_eb = L->routed.w13_expert_bytes;
  ga.tile_r = w13_tile_bytes(L->routed.fmt, H);
  ga.s_base = L->shared.w13;
  ga.tile_s = fp8_w13_tile_bytes(H);
  ga.KC_r8 = H / 32;
  ga.KC_s = H / 32;
  ga.chunks = g.chunks;
  ga.nchunks = g.nchunks;
  ga.bsrc = ws + w.bbuf1;
  ga.katoms = H / 128;
  ga.mtiles = I / 64;
  ga.out = (float*)(ws + w.gu);
  ga.out_ld = 2 * I;
  ga.pair_tok = g.pair_tok;
  ga.xscale = (const float*)(ws + w.xscale);
  ga.status = status;
  prefill_gemm_kernel<<<sms, PFT, PSMEM, st>>>(ga);

  ta.dst = ws + w.bbuf2;
  prefill_rows_kernel<2><<<maxc, 256, 0, st>>>(ta);

  GemmArgs gb = ga;
  gb.phase = 2;
  gb.r_base = L->routed.w2;
  gb.r_eb = L->routed.w2_expert_bytes;
  gb.tile_r = w2_tile_bytes(L->routed.fmt, I);
  gb.s_base = L->shared.w2;
  gb.tile_s = fp8_w2_tile_bytes(I);
  gb.KC_r8 = I / 32;
  gb.KC_s = I / 32;
  gb.bsrc = ws + w.bbuf2;
  gb.katoms = I / 128;
  gb.mtiles = H / 128;
  gb.out = (float*)(ws + w.ypair);
  gb.out_ld = H;
  prefill_gemm_kernel<<<sms, PFT, PSMEM, st>>>(gb);

  prefill_combine_kernel<<<dim3((H + 255) / 256, P), 256, 0, st>>>((const float*)(ws + w.ypair), g.pos_of, wt, P, K, H,
                                                                  y, y_dtype == DSMOE_DTYPE_F32);
  return cuda_status("prefill");
}

extern "C" int dsmoe_moe_prefill_check(const dsmoe_layer_t* L, int P, void* workspace, size_t workspace_bytes,
                                       void* stream) {
  int rc = prefill_validate(L, P);
  if (rc) return rc;
  const PrefillWs w = prefill_ws(P, L->hidden, L->inter_local, L->n_experts, L->topk);
  DSMOE_REQUIRE(workspace && workspace_bytes >= w.total, DSMOE_ERR_WORKSPACE, "prefill_check: workspace too small");
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaStreamSynchronize(st) != cudaSuccess) return cuda_status("prefill_check: synchronize");
  unsigned status = 0;
  if (cudaMemcpy(&status, (uint8_t*)workspace + w.status, 4, cudaMemcpyDeviceToHost) != cudaSuccess)
    return cuda_status("prefill_check: read status");
  if (status == 0) return DSMOE_OK;
  cudaMemset((uint8_t*)workspace + w.status, 0, 4);
  set_error("prefill: %s (status 0x%x)", (status & PST_ROUTE) ? "an expert index was out of range"
                                                              : "a bounded device wait expired", status);
  return (status & PST_ROUTE) ? DSMOE_ERR_ARG : DSMOE_ERR_TIMEOUT;
}
