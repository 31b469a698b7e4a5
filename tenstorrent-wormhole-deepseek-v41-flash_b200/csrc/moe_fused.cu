// One persistent kernel per MoE layer for decode batches of 1..8 tokens.
//
// Replaces the per-layer sequence of the reference's decode -- device router GEMV, host top-k,
// host->device control write, SlotCat gather, w1/w3/shared matmuls, Q20 SwiGLU, w2 matmuls
// (dsv41/tt/model.py:400-442; dsv41/tt/moe.py:108-180; dsv41/kernels/slot_cat.cpp) -- with one
// launch that streams every weight byte the step needs exactly once.
//
// Shape: one CTA per SM (cooperative launch), 8 consumer warps + 1 producer warp.
//   producer   one thread issues 1-D bulk copies (cp.async.bulk, the TMA engine) of each work
//              item's weight bytes into a ring of up to 16 x 8.5 KB shared-memory stages,
//              completion counted on per-stage mbarriers; it runs ahead across phase boundaries
//              (w2 weights stream in while the grid waits for the last w1|w3 tiles).
//   consumers  each item is consumed by one warp: dequantize the A fragments from the stage,
//              mma.sync m16n8k16 (f16 x f16 -> fp32) against the tokens' f16 fragments (shared
//              memory), block scales on the fp32 partials, partial sums to global scratch.
// Phases (items are dealt round-robin over the CTAs, rotating across phases so every CTA gets the
// same amount of work):
//   R  router quarter-rows (fp64 accumulation) + the shared expert's w1|w3 parts (no routing
//      needed); a CTA arrives at grid barrier A as soon as its router items are done, so the
//      shared-expert work hides the barrier.
//   P  every CTA computes the same top-k and slot plan from the router partials (no extra barrier).
//   1  routed w1|w3 parts. The last part of each 16-row tile (a counter) sums the tile's partials
//      in a fixed order and applies clamp / SiLU / up / routing weight -> h (f16).
//   2  (after grid barrier B) w2 parts per 16 output rows x slot x K range; the last part of each
//      16-row tile sums the partials in a fixed order -> y. Results are deterministic.
// Every wait (mbarrier, grid barrier) is bounded by %globaltimer; on expiry the kernel records a
// status bit in the workspace, stops issuing work, lets its own copies land and returns.
#include "router.cuh"

namespace dsmoe {

constexpr int FW = 8;                  // consumer warps
constexpr int FT = (FW + 1) * 32;      // + producer warp
constexpr int FCH = 8;                 // packed chunks per w1|w3 or w2 item
constexpr int FSTAGE = FCH * 1088;     // bytes per ring stage (8 FP4 w1|w3 chunks, the largest item)
constexpr int FMAXB = 8;               // tokens per call
constexpr int FMAXK = DSMOE_MAX_TOPK;
constexpr int FMAXS = FMAXB * FMAXK + 1;
constexpr int FEMAX = 1024;            // routed experts
constexpr uint64_t kWaitNs = 1000000000ull;

enum : unsigned { ST_FULL = 1u, ST_EMPTY = 2u, ST_PLAN = 4u, ST_GRID = 8u };

struct FusedArgs {
  int H, I_loc, E, B, topk, score_func;
  float route_scale;
  const float* wg;
  const float* bias;
  const float* bias_vl;
  const uint8_t* image_mask;
  const __nv_bfloat16* x;
  int r_fmt;
  const uint8_t* r_w13;
  const uint8_t* r_w2;
  long long r_w13_eb, r_w2_eb;
  const uint8_t* s_w13;
  const uint8_t* s_w2;
  void* y;
  int y_f32;
  int64_t* idx;
  float* wt;
  float* scores;
  // scratch (workspace)
  double* rl;        // [B][E][4] router quarter-row partial logits
  float* p13;        // [slots][T][p13max][32][8] w1|w3 partials
  float* p2;         // [NT][qmax][32][4] w2 partials (token columns)
  uint16_t* hf;      // [slots * 8][I_loc] h, f16, fragment order
  unsigned* cnt13;   // [slots][T]
  unsigned* cnt2;    // [NT]
  unsigned* gbar;    // [0] arrivals, [1] generation
  unsigned* status;  // [0]
  int sh_idx;        // scratch slot index of the shared expert (= B * topk)
  int nstage, xrow, p13max, qmax;
};

struct FPlan {
  int n_routed;
  int expert[FMAXS];
  int ntok[FMAXS];
  int tok[FMAXS][8];
  float wt[FMAXS][8];
  signed char col_of[FMAXS][8];
  float xscale[FMAXB];
  int sel[FMAXB][FMAXK];
  float selw[FMAXB][FMAXK];
  int wcnt[FW];
  unsigned router_done;
  unsigned gen_a;
  int abort;
};

struct Geo {
  int T, NT, KB, NR, NS, P13s, P13r, KC2s, KC2r, P2s, P2r;
  int chunk13r, chunk2r;
  long long tile13r, tile13s, tile2r, tile2s;
};

__device__ __forceinline__ Geo make_geo(const FusedArgs& a) {
  Geo g;
  g.T = a.I_loc / 16;
  g.NT = a.H / 16;
  g.KB = a.H / 128;
  g.NR = 4 * a.E;
  g.P13s = (a.H / 32) / FCH;
  g.P13r = a.r_fmt == DSMOE_FMT_FP8 ? (a.H / 32) / FCH : (a.H / 64) / FCH;
  g.NS = g.T * g.P13s;
  g.KC2s = a.I_loc / 32;
  g.KC2r = a.r_fmt == DSMOE_FMT_FP8 ? a.I_loc / 32 : a.I_loc / 64;
  g.P2s = (g.KC2s + FCH - 1) / FCH;
  g.P2r = (g.KC2r + FCH - 1) / FCH;
  g.chunk13r = a.r_fmt == DSMOE_FMT_FP8 ? 1024 : 1088;
  g.chunk2r = a.r_fmt == DSMOE_FMT_FP8 ? 512 : 544;
  g.tile13r = w13_tile_bytes(a.r_fmt, a.H);
  g.tile13s = fp8_w13_tile_bytes(a.H);
  g.tile2r = w2_tile_bytes(a.r_fmt, a.I_loc);
  g.tile2s = fp8_w2_tile_bytes(a.I_loc);
  return g;
}

// first item of CTA c in a phase whose items are dealt from CTA (base % G)
__device__ __forceinline__ int first_item(int base, int c, int G) {
  int f = c - base % G;
  return f < 0 ? f + G : f;
}

__device__ __forceinline__ float fscore(float l, int func) {
  const double d = (double)l;
  const double s = func == DSMOE_SCORE_SIGMOID ? 1.0 / (1.0 + exp(-d)) : sqrt(d > 20.0 ? d : log1p(exp(d)));
  return __double2float_rn(s);
}

__device__ __forceinline__ uint4 lds16(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }

__device__ __forceinline__ int frag_pos(int j) {
  const int k = j & 31, s = k >> 4, kk = k & 15;
  return (j >> 5) * 32 + ((kk & 7) >> 1) * 8 + (2 * s + (kk >> 3)) * 2 + (kk & 1);
}

__device__ __forceinline__ void fma4s(float (&acc)[4], float (&t)[4], float s) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    acc[j] = fmaf(t[j], s, acc[j]);
    t[j] = 0.f;
  }
}
__device__ __forceinline__ void fma4r(float (&acc)[4], float (&t)[4], float s_lo, float s_hi) {
  acc[0] = fmaf(t[0], s_lo, acc[0]);
  acc[1] = fmaf(t[1], s_lo, acc[1]);
  acc[2] = fmaf(t[2], s_hi, acc[2]);
  acc[3] = fmaf(t[3], s_hi, acc[3]);
#pragma unroll
  for (int j = 0; j < 4; ++j) t[j] = 0.f;
}

// ------------------------------------------------------------------ grid barrier (bounded)
__device__ __forceinline__ unsigned grid_arrive(unsigned* gbar, int G) {
  const unsigned g0 = ld_acquire_u32(gbar + 1);
  __threadfence();
  const unsigned old = atomicAdd(gbar, 1u);
  if (old == (unsigned)G - 1) {
    atomicExch(gbar, 0u);
    __threadfence();
    atomicAdd(gbar + 1, 1u);
  }
  return g0;
}
__device__ __forceinline__ bool grid_wait(unsigned* gbar, unsigned g0, const unsigned* status) {
  const uint64_t t0 = globaltimer_ns();
  while (ld_acquire_u32(gbar + 1) == g0) {
    if (ld_acquire_u32(status) != 0u) return false;
    if (globaltimer_ns() - t0 > kWaitNs) return false;
    __nanosleep(64);
  }
  return true;
}

// ------------------------------------------------------------------ items (one warp each)
// Router quarter-row: 1/4 of gate_w[r] (H/4 fp32, in the stage) . x[b] for every token, fp64.
__device__ void router_item(const FusedArgs& a, const uint8_t* stage, int r, int q, int lane) {
  double acc[FMAXB];
#pragma unroll
  for (int b = 0; b < FMAXB; ++b) acc[b] = 0.0;
  const float4* wv = reinterpret_cast<const float4*>(stage);
  const int n4 = a.H / 16;  // float4 per quarter
  for (int f = lane; f < n4; f += 32) {
    const float4 w = wv[f];
    const int k = q * (a.H / 4) + 4 * f;
#pragma unroll
    for (int b = 0; b < FMAXB; ++b) {
      if (b < a.B) {
        const uint2 xv = __ldg(reinterpret_cast<const uint2*>(a.x + (long long)b * a.H + k));
        acc[b] = fma((double)__uint_as_float(xv.x << 16), (double)w.x, acc[b]);
        acc[b] = fma((double)__uint_as_float(xv.x & 0xFFFF0000u), (double)w.y, acc[b]);
        acc[b] = fma((double)__uint_as_float(xv.y << 16), (double)w.z, acc[b]);
        acc[b] = fma((double)__uint_as_float(xv.y & 0xFFFF0000u), (double)w.w, acc[b]);
      }
    }
  }
#pragma unroll
  for (int b = 0; b < FMAXB; ++b) {
    if (b < a.B) {
      const double v = warp_sum_d(acc[b]);
      if (lane == 0) a.rl[((long long)b * a.E + r) * 4 + q] = v;
    }
  }
}

// Sum a w1|w3 tile's partials in order and write h (clamp, SiLU, up, routing weight).
__device__ void finalize_w13(const FusedArgs& a, const Geo& G, const FPlan& pl, int sidx, int t, int nparts,
                             int ntok, const int* toks, const float* wts, int lane) {
  float s[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) s[j] = 0.f;
  for (int q = 0; q < nparts; ++q) {
    const float* src = a.p13 + ((((long long)sidx * G.T + t) * a.p13max + q) * 32 + lane) * 8;
    const uint4 v0 = ld_cg16(src), v1 = ld_cg16(src + 4);
    s[0] += __uint_as_float(v0.x); s[1] += __uint_as_float(v0.y);
    s[2] += __uint_as_float(v0.z); s[3] += __uint_as_float(v0.w);
    s[4] += __uint_as_float(v1.x); s[5] += __uint_as_float(v1.y);
    s[6] += __uint_as_float(v1.z); s[7] += __uint_as_float(v1.w);
  }
  const int g = lane >> 2, tq = lane & 3;
#pragma unroll
  for (int q4 = 0; q4 < 4; ++q4) {
    const int row = q4 >= 2 ? g + 8 : g, col = 2 * tq + (q4 & 1);
    if (col < ntok) {
      const float xs = pl.xscale[toks[col]];
      const float gv = fminf(s[q4] * xs, 10.0f);
      const float uv = fminf(fmaxf(s[4 + q4] * xs, -10.0f), 10.0f);
      const float h = silu_f(gv) * uv * wts[col];
      a.hf[(long long)(sidx * 8 + col) * a.I_loc + frag_pos(16 * t + row)] = __half_as_ushort(__float2half_rn(h));
    }
  }
}

// One w1|w3 item: 8 chunks of a 16-row tile against the slot's tokens.
template <int FMT>
__device__ void w13_item(const FusedArgs& a, const Geo& G, const FPlan& pl, const uint8_t* stage, const uint8_t* xf,
                         const uint8_t* tile_g, int sidx, int t, int p, int nparts, int ntok, const int* toks,
                         const float* wts, int lane) {
  const int g = lane >> 2, tq = lane & 3;
  const uint8_t* xrow = xf + (long long)toks[min(g, ntok - 1)] * a.xrow;
  float acc1[4] = {0.f, 0.f, 0.f, 0.f}, acc3[4] = {0.f, 0.f, 0.f, 0.f};
  float t1[4] = {0.f, 0.f, 0.f, 0.f}, t3[4] = {0.f, 0.f, 0.f, 0.f};
  if (FMT == DSMOE_FMT_FP8) {
    const float* sc = reinterpret_cast<const float*>(tile_g + (long long)(a.H / 32) * 1024);
#pragma unroll
    for (int c = 0; c < FCH; ++c) {
      const int gc = p * FCH + c;
      const uint4 A1 = lds16(stage + c * 1024 + lane * 16);
      const uint4 A3 = lds16(stage + c * 1024 + 512 + lane * 16);
      const uint4 X = lds16(xrow + gc * 64 + tq * 16);
      uint32_t A[4];
      a_frag_fp8(A, A1.x, A1.y); mma16816(t1, A, X.x, X.y);
      a_frag_fp8(A, A3.x, A3.y); mma16816(t3, A, X.x, X.y);
      a_frag_fp8(A, A1.z, A1.w); mma16816(t1, A, X.z, X.w);
      a_frag_fp8(A, A3.z, A3.w); mma16816(t3, A, X.z, X.w);
      if ((c & 3) == 3) {
        const int kb = gc >> 2;
        fma4s(acc1, t1, __ldg(sc + kb));
        fma4s(acc3, t3, __ldg(sc + G.KB + kb));
      }
    }
  } else {
#pragma unroll
    for (int c = 0; c < FCH; ++c) {
      const int gc = p * FCH + c;
      const uint8_t* ch = stage + c * 1088;
      const uint4 A1 = lds16(ch + lane * 16), A3 = lds16(ch + 512 + lane * 16);
      const uint32_t S1 = lds32(ch + 1024 + 4 * g), S3 = lds32(ch + 1056 + 4 * g);
      const uint4 X0 = lds16(xrow + (2 * gc) * 64 + tq * 16), X1 = lds16(xrow + (2 * gc + 1) * 64 + tq * 16);
      uint32_t A[4];
      a_frag_fp4(A, A1.x); mma16816(t1, A, X0.x, X0.y);
      a_frag_fp4(A, A1.y); mma16816(t1, A, X0.z, X0.w);
      a_frag_fp4(A, A3.x); mma16816(t3, A, X0.x, X0.y);
      a_frag_fp4(A, A3.y); mma16816(t3, A, X0.z, X0.w);
      fma4r(acc1, t1, e8m0_to_f32(S1), e8m0_to_f32(S1 >> 16));
      fma4r(acc3, t3, e8m0_to_f32(S3), e8m0_to_f32(S3 >> 16));
      a_frag_fp4(A, A1.z); mma16816(t1, A, X1.x, X1.y);
      a_frag_fp4(A, A1.w); mma16816(t1, A, X1.z, X1.w);
      a_frag_fp4(A, A3.z); mma16816(t3, A, X1.x, X1.y);
      a_frag_fp4(A, A3.w); mma16816(t3, A, X1.z, X1.w);
      fma4r(acc1, t1, e8m0_to_f32(S1 >> 8), e8m0_to_f32(S1 >> 24));
      fma4r(acc3, t3, e8m0_to_f32(S3 >> 8), e8m0_to_f32(S3 >> 24));
    }
  }
  float* dst = a.p13 + ((((long long)sidx * G.T + t) * a.p13max + p) * 32 + lane) * 8;
  *reinterpret_cast<float4*>(dst) = make_float4(acc1[0], acc1[1], acc1[2], acc1[3]);
  *reinterpret_cast<float4*>(dst + 4) = make_float4(acc3[0], acc3[1], acc3[2], acc3[3]);
  __threadfence();
  __syncwarp();
  unsigned old = 0;
  if (lane == 0) old = atomicAdd(a.cnt13 + sidx * G.T + t, 1u);
  old = __shfl_sync(0xffffffffu, old, 0);
  if (old == (unsigned)nparts - 1) {
    __threadfence();
    finalize_w13(a, G, pl, sidx, t, nparts, ntok, toks, wts, lane);
    if (lane == 0) a.cnt13[sidx * G.T + t] = 0u;
  }
}

// One w2 item: up to 8 chunks of one slot's 16 output rows x K range; partial in token columns.
template <int FMT>
__device__ void w2_item(const FusedArgs& a, const Geo& G, const FPlan& pl, const uint8_t* stage,
                        const uint8_t* tile_g, int s, int sidx, int nt, int p, int nch, int q, int Q, int lane) {
  const int g = lane >> 2, tq = lane & 3;
  const uint8_t* hrow = reinterpret_cast<const uint8_t*>(a.hf + (long long)(sidx * 8 + g) * a.I_loc) + tq * 16;
  float acc[4] = {0.f, 0.f, 0.f, 0.f}, tt[4] = {0.f, 0.f, 0.f, 0.f};
  if (FMT == DSMOE_FMT_FP8) {
    const int KC = a.I_loc / 32;
    const float* sc = reinterpret_cast<const float*>(tile_g + (long long)KC * 512);
    uint4 hb[FCH];
#pragma unroll
    for (int i = 0; i < FCH; ++i)
      if (i < nch) hb[i] = ld_cg16(hrow + (long long)(p * FCH + i) * 64);
#pragma unroll
    for (int i = 0; i < FCH; ++i) {
      if (i < nch) {
        const uint4 A0 = lds16(stage + i * 512 + lane * 16);
        uint32_t A[4];
        a_frag_fp8(A, A0.x, A0.y); mma16816(tt, A, hb[i].x, hb[i].y);
        a_frag_fp8(A, A0.z, A0.w); mma16816(tt, A, hb[i].z, hb[i].w);
        fma4s(acc, tt, __ldg(sc + p * FCH + i));
      }
    }
  } else {
    uint4 hb[2 * FCH];
#pragma unroll
    for (int i = 0; i < FCH; ++i) {
      if (i < nch) {
        hb[2 * i] = ld_cg16(hrow + (long long)(2 * (p * FCH + i)) * 64);
        hb[2 * i + 1] = ld_cg16(hrow + (long long)(2 * (p * FCH + i) + 1) * 64);
      }
    }
#pragma unroll
    for (int i = 0; i < FCH; ++i) {
      if (i < nch) {
        const uint8_t* ch = stage + i * 544;
        const uint4 A0 = lds16(ch + lane * 16);
        const uint32_t S = lds32(ch + 512 + 4 * g);
        uint32_t A[4];
        a_frag_fp4(A, A0.x); mma16816(tt, A, hb[2 * i].x, hb[2 * i].y);
        a_frag_fp4(A, A0.y); mma16816(tt, A, hb[2 * i].z, hb[2 * i].w);
        fma4r(acc, tt, e8m0_to_f32(S), e8m0_to_f32(S >> 16));
        a_frag_fp4(A, A0.z); mma16816(tt, A, hb[2 * i + 1].x, hb[2 * i + 1].y);
        a_frag_fp4(A, A0.w); mma16816(tt, A, hb[2 * i + 1].z, hb[2 * i + 1].w);
        fma4r(acc, tt, e8m0_to_f32(S >> 8), e8m0_to_f32(S >> 24));
      }
    }
  }
  // slot columns -> token columns: lane (g, tq) collects tokens 2tq, 2tq+1 of rows g, g+8
  float out[4];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int tok = 2 * tq + h;
    const int col = tok < a.B ? pl.col_of[s][tok] : -1;
    const int src = g * 4 + (col < 0 ? 0 : col >> 1);
    const float v0 = __shfl_sync(0xffffffffu, acc[0], src), v1 = __shfl_sync(0xffffffffu, acc[1], src);
    const float v2 = __shfl_sync(0xffffffffu, acc[2], src), v3 = __shfl_sync(0xffffffffu, acc[3], src);
    out[h] = col < 0 ? 0.f : ((col & 1) ? v1 : v0);
    out[2 + h] = col < 0 ? 0.f : ((col & 1) ? v3 : v2);
  }
  float* dst = a.p2 + (((long long)nt * a.qmax + q) * 32 + lane) * 4;
  *reinterpret_cast<float4*>(dst) = make_float4(out[0], out[1], out[2], out[3]);
  __threadfence();
  __syncwarp();
  unsigned old = 0;
  if (lane == 0) old = atomicAdd(a.cnt2 + nt, 1u);
  old = __shfl_sync(0xffffffffu, old, 0);
  if (old == (unsigned)Q - 1) {
    __threadfence();
    float sum[4] = {0.f, 0.f, 0.f, 0.f};
    for (int qq = 0; qq < Q; ++qq) {
      const uint4 v = ld_cg16(a.p2 + (((long long)nt * a.qmax + qq) * 32 + lane) * 4);
      sum[0] += __uint_as_float(v.x); sum[1] += __uint_as_float(v.y);
      sum[2] += __uint_as_float(v.z); sum[3] += __uint_as_float(v.w);
    }
#pragma unroll
    for (int q4 = 0; q4 < 4; ++q4) {
      const int row = nt * 16 + (q4 >= 2 ? g + 8 : g), tok = 2 * tq + (q4 & 1);
      if (tok < a.B) {
        const long long o = (long long)tok * a.H + row;
        if (a.y_f32)
          reinterpret_cast<float*>(a.y)[o] = sum[q4];
        else
          reinterpret_cast<__nv_bfloat16*>(a.y)[o] = __float2bfloat16_rn(sum[q4]);
      }
    }
    if (lane == 0) a.cnt2[nt] = 0u;
  }
}

// ------------------------------------------------------------------ the kernel
template <int RFMT>
__global__ void __launch_bounds__(FT, 1) moe_fused_kernel(FusedArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ring = smem;
  uint8_t* xf = ring + (size_t)a.nstage * FSTAGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(xf + (size_t)a.B * a.xrow);
  uint64_t* empty = full + a.nstage;
  uint64_t* planbar = empty + a.nstage;
  FPlan& pl = *reinterpret_cast<FPlan*>(planbar + 2);
  unsigned* emask = reinterpret_cast<unsigned*>(&pl + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int G = gridDim.x, cta = blockIdx.x;
  const Geo geo = make_geo(a);
  const int nR = geo.NR + geo.NS;
  int my_router = 0;
  for (int i = first_item(0, cta, G); i < geo.NR; i += G) ++my_router;

  if (tid == 0) {
    for (int s = 0; s < a.nstage; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(planbar, 1);
    pl.router_done = 0;
    pl.abort = 0;
    fence_mbar_init();
  }
  __syncthreads();

  // ================================================================ producer warp
  if (warp == FW) {
    if (lane != 0) return;
    int j = 0;
    bool ok = true;
    auto issue = [&](const void* src, uint32_t bytes) {
      if (!ok) return;
      const int s = j % a.nstage, k = j / a.nstage;
      if (k > 0 && !mbar_wait(&empty[s], (k - 1) & 1, kWaitNs)) {
        atomicOr(a.status, ST_EMPTY);
        ok = false;
        return;
      }
      mbar_expect_tx(&full[s], bytes);
      bulk_g2s(ring + (size_t)s * FSTAGE, src, bytes, &full[s]);
      ++j;
    };
    for (int i = first_item(0, cta, G); i < nR && ok; i += G) {
      if (i < geo.NR) {
        issue(a.wg + (long long)(i >> 2) * a.H + (i & 3) * (a.H / 4), (uint32_t)a.H);
      } else {
        const int i2 = i - geo.NR, t = i2 / geo.P13s, p = i2 % geo.P13s;
        issue(a.s_w13 + t * geo.tile13s + (long long)p * FCH * 1024, FCH * 1024);
      }
    }
    if (ok && !mbar_wait(planbar, 0, 4 * kWaitNs)) {
      atomicOr(a.status, ST_PLAN);
      ok = false;
    }
    if (ok) {
      const int nr = pl.n_routed;
      const int N1 = nr * geo.T * geo.P13r;
      for (int i = first_item(nR, cta, G); i < N1 && ok; i += G) {
        const int per = geo.T * geo.P13r, s = i / per, rem = i % per, t = rem / geo.P13r, p = rem % geo.P13r;
        const uint8_t* base = a.r_w13 + (long long)pl.expert[s] * a.r_w13_eb + t * geo.tile13r;
        issue(base + (long long)p * FCH * geo.chunk13r, (uint32_t)(FCH * geo.chunk13r));
      }
      const int Q = nr * geo.P2r + geo.P2s;
      const int N2 = geo.NT * Q;
      for (int i = first_item(nR + N1, cta, G); i < N2 && ok; i += G) {
        const int nt = i / Q, jq = i % Q;
        const uint8_t* src;
        uint32_t bytes;
        if (jq < nr * geo.P2r) {
          const int s = jq / geo.P2r, p = jq % geo.P2r;
          const int nch = min(FCH, geo.KC2r - p * FCH);
          src = a.r_w2 + (long long)pl.expert[s] * a.r_w2_eb + nt * geo.tile2r + (long long)p * FCH * geo.chunk2r;
          bytes = (uint32_t)(nch * geo.chunk2r);
        } else {
          const int p = jq - nr * geo.P2r, nch = min(FCH, geo.KC2s - p * FCH);
          src = a.s_w2 + nt * geo.tile2s + (long long)p * FCH * 512;
          bytes = (uint32_t)(nch * 512);
        }
        issue(src, bytes);
      }
    }
    // let every copy this thread issued land before the CTA may exit
    for (int jj = max(0, j - a.nstage); jj < j; ++jj) mbar_wait(&full[jj % a.nstage], (jj / a.nstage) & 1, kWaitNs);
    return;
  }

  // ================================================================ consumer warps
  // token fragments: amax -> power-of-2 pre-scale -> f16 fragments in shared memory
  if (warp < a.B) {
    const __nv_bfloat16* xr = a.x + (long long)warp * a.H;
    float m = 0.f;
    for (int i = lane * 8; i < a.H; i += 256) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(xr + i));
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int h = 0; h < 4; ++h)
        m = fmaxf(m, fmaxf(fabsf(__uint_as_float(w[h] << 16)), fabsf(__uint_as_float(w[h] & 0xFFFF0000u))));
    }
    m = warp_max(m);
    int p = 0;
    if (m > 0.f && m <= 3.0e38f) {
      int e2;
      frexpf(m, &e2);
      p = e2 - 15;
    }
    if (lane == 0) pl.xscale[warp] = ldexpf(1.0f, p);
    const float inv = ldexpf(1.0f, -p);
    for (int i = lane; i < (a.H / 32) * 4; i += 32) {
      const int c = i >> 2, tq = i & 3, k0 = 32 * c + 2 * tq;
      auto pr = [&](int k) {
        return pack_f16x2(__bfloat162float(xr[k]) * inv, __bfloat162float(xr[k + 1]) * inv);
      };
      *reinterpret_cast<uint4*>(xf + (long long)warp * a.xrow + c * 64 + tq * 16) =
          make_uint4(pr(k0), pr(k0 + 8), pr(k0 + 16), pr(k0 + 24));
    }
  }
  for (int e = tid; e < a.E; e += FW * 32) emask[e] = 0u;
  if (my_router == 0 && tid == 0) pl.gen_a = grid_arrive(a.gbar, G);
  named_bar_sync(1, FW * 32);

  int shared_toks[FMAXB];
  float shared_wts[FMAXB];
#pragma unroll
  for (int b = 0; b < FMAXB; ++b) {
    shared_toks[b] = min(b, a.B - 1);
    shared_wts[b] = 1.0f;
  }

  int j = 0;  // CTA item sequence (same order as the producer)
  auto wait_full = [&](int jj) -> bool {
    if (*(volatile int*)&pl.abort) return false;
    if (!mbar_wait(&full[jj % a.nstage], (jj / a.nstage) & 1, kWaitNs)) {
      if (lane == 0) {
        atomicOr(a.status, ST_FULL);
        pl.abort = 1;
      }
      return false;
    }
    return true;
  };
  auto release = [&](int jj) {
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[jj % a.nstage]);
  };

  // ---- phase R: router quarter-rows, then the shared expert's w1|w3 parts
  for (int i = first_item(0, cta, G); i < nR; i += G, ++j) {
    if (j % FW != warp) continue;
    if (!wait_full(j)) break;
    const uint8_t* stage = ring + (size_t)(j % a.nstage) * FSTAGE;
    if (i < geo.NR) {
      router_item(a, stage, i >> 2, i & 3, lane);
      release(j);
      __threadfence();
      __syncwarp();
      if (lane == 0) {
        const unsigned done = atomicAdd(&pl.router_done, 1u) + 1;
        if ((int)done == my_router) pl.gen_a = grid_arrive(a.gbar, G);
      }
    } else {
      const int i2 = i - geo.NR, t = i2 / geo.P13s, p = i2 % geo.P13s;
      w13_item<DSMOE_FMT_FP8>(a, geo, pl, stage, xf, a.s_w13 + t * geo.tile13s, a.sh_idx, t, p, geo.P13s, a.B,
                              shared_toks, shared_wts, lane);
      release(j);
    }
  }
  __threadfence();
  named_bar_sync(1, FW * 32);
  if (tid == 0 && !pl.abort) {
    if (!grid_wait(a.gbar, pl.gen_a, a.status)) {
      atomicOr(a.status, ST_GRID);
      pl.abort = 1;
    }
  }
  named_bar_sync(1, FW * 32);
  if (pl.abort) return;

  // ---- plan: identical in every CTA
  if (warp < a.B) {
    const int b = warp;
    float scv[FEMAX / 32], biv[FEMAX / 32];
    const bool vl = a.bias_vl != nullptr && a.image_mask != nullptr && a.image_mask[b] != 0;
    const float* bias = vl ? a.bias_vl : a.bias;
#pragma unroll
    for (int i = 0; i < FEMAX / 32; ++i) {
      const int e = lane + 32 * i;
      scv[i] = 0.f;
      biv[i] = -INFINITY;
      if (e < a.E) {
        const double* r4 = a.rl + ((long long)b * a.E + e) * 4;
        const double l = ((ld_cg_f64(r4) + ld_cg_f64(r4 + 1)) + ld_cg_f64(r4 + 2)) + ld_cg_f64(r4 + 3);
        const float sc = fscore(__double2float_rn(l), a.score_func);
        scv[i] = sc;
        biv[i] = sc + bias[e];
        if (cta == 0 && a.scores) a.scores[(long long)b * a.E + e] = sc;
      }
    }
    float tot = 0.f;
    for (int r = 0; r < a.topk; ++r) {
      float best = -INFINITY;
      int bi = 0x7FFFFFFF;
#pragma unroll
      for (int i = 0; i < FEMAX / 32; ++i) {
        const int e = lane + 32 * i;
        if (e < a.E && (biv[i] > best || (biv[i] == best && e < bi))) {
          best = biv[i];
          bi = e;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > best || (ov == best && oi < bi)) {
          best = ov;
          bi = oi;
        }
      }
      if (bi == 0x7FFFFFFF) bi = 0;
      float scw = 0.f;
#pragma unroll
      for (int i = 0; i < FEMAX / 32; ++i) {
        if (lane + 32 * i == bi) {
          scw = scv[i];
          biv[i] = -INFINITY;
        }
      }
      scw = __shfl_sync(0xffffffffu, scw, bi & 31);
      if (lane == 0) {
        pl.sel[b][r] = bi;
        pl.selw[b][r] = scw;
      }
      tot += scw;
    }
    if (lane == 0) {
      for (int r = 0; r < a.topk; ++r) {
        const float w = pl.selw[b][r] / (tot + 1e-20f) * a.route_scale;
        pl.selw[b][r] = w;
        if (cta == 0) {
          if (a.idx) a.idx[b * a.topk + r] = pl.sel[b][r];
          if (a.wt) a.wt[b * a.topk + r] = w;
        }
      }
    }
  }
  named_bar_sync(1, FW * 32);
  for (int i = tid; i < a.B * a.topk; i += FW * 32) atomicOr(&emask[pl.sel[i / a.topk][i % a.topk]], 1u << (i / a.topk));
  named_bar_sync(1, FW * 32);
  {
    int base = 0;
    for (int e0 = 0; e0 < a.E; e0 += FW * 32) {
      const int e = e0 + tid;
      const unsigned m = e < a.E ? emask[e] : 0u;
      const unsigned bal = __ballot_sync(0xffffffffu, m != 0u);
      if (lane == 0) pl.wcnt[warp] = __popc(bal);
      named_bar_sync(1, FW * 32);
      int off = base, total = 0;
      for (int w = 0; w < FW; ++w) {
        if (w < warp) off += pl.wcnt[w];
        total += pl.wcnt[w];
      }
      off += __popc(bal & ((1u << lane) - 1u));
      if (m != 0u) {
        pl.expert[off] = e;
        pl.ntok[off] = __popc(m);
        int n = 0;
        for (int b = 0; b < FMAXB; ++b) pl.col_of[off][b] = -1;
        for (int b = 0; b < a.B; ++b) {
          if (m & (1u << b)) {
            float w = 0.f;
            for (int r = 0; r < a.topk; ++r)
              if (pl.sel[b][r] == e) w = pl.selw[b][r];
            pl.tok[off][n] = b;
            pl.wt[off][n] = w;
            pl.col_of[off][b] = (signed char)n;
            ++n;
          }
        }
        for (; n < 8; ++n) {
          pl.tok[off][n] = pl.tok[off][0];
          pl.wt[off][n] = 0.f;
        }
      }
      base += total;
      named_bar_sync(1, FW * 32);
    }
    if (tid == 0) {
      const int s = base;  // the shared expert's slot
      pl.n_routed = base;
      pl.expert[s] = a.E;
      pl.ntok[s] = a.B;
      for (int b = 0; b < 8; ++b) {
        pl.tok[s][b] = min(b, a.B - 1);
        pl.wt[s][b] = 1.0f;
        pl.col_of[s][b] = b < a.B ? (signed char)b : (signed char)-1;
      }
    }
  }
  named_bar_sync(1, FW * 32);
  if (tid == 0) mbar_arrive(planbar);

  // ---- phase 1: routed w1|w3
  const int nr = pl.n_routed;
  const int N1 = nr * geo.T * geo.P13r;
  for (int i = first_item(nR, cta, G); i < N1; i += G, ++j) {
    if (j % FW != warp) continue;
    if (!wait_full(j)) break;
    const uint8_t* stage = ring + (size_t)(j % a.nstage) * FSTAGE;
    const int per = geo.T * geo.P13r, s = i / per, rem = i % per, t = rem / geo.P13r, p = rem % geo.P13r;
    const uint8_t* tile_g = a.r_w13 + (long long)pl.expert[s] * a.r_w13_eb + t * geo.tile13r;
    w13_item<RFMT>(a, geo, pl, stage, xf, tile_g, s, t, p, geo.P13r, pl.ntok[s], pl.tok[s], pl.wt[s], lane);
    release(j);
  }
  __threadfence();
  named_bar_sync(1, FW * 32);
  if (tid == 0 && !pl.abort) {
    const unsigned g0 = grid_arrive(a.gbar, G);
    if (!grid_wait(a.gbar, g0, a.status)) {
      atomicOr(a.status, ST_GRID);
      pl.abort = 1;
    }
  }
  named_bar_sync(1, FW * 32);
  if (pl.abort) return;

  // ---- phase 2: w2
  const int Q = nr * geo.P2r + geo.P2s;
  const int N2 = geo.NT * Q;
  for (int i = first_item(nR + N1, cta, G); i < N2; i += G, ++j) {
    if (j % FW != warp) continue;
    if (!wait_full(j)) break;
    const uint8_t* stage = ring + (size_t)(j % a.nstage) * FSTAGE;
    const int nt = i / Q, jq = i % Q;
    if (jq < nr * geo.P2r) {
      const int s = jq / geo.P2r, p = jq % geo.P2r, nch = min(FCH, geo.KC2r - p * FCH);
      const uint8_t* tile_g = a.r_w2 + (long long)pl.expert[s] * a.r_w2_eb + nt * geo.tile2r;
      w2_item<RFMT>(a, geo, pl, stage, tile_g, s, s, nt, p, nch, jq, Q, lane);
    } else {
      const int p = jq - nr * geo.P2r, nch = min(FCH, geo.KC2s - p * FCH);
      w2_item<DSMOE_FMT_FP8>(a, geo, pl, stage, a.s_w2 + nt * geo.tile2s, nr, a.sh_idx, nt, p, nch, jq, Q, lane);
    }
    release(j);
  }
}

// ------------------------------------------------------------------ host side
size_t fused_smem_bytes(int H, int B, int E, int nstage) {
  const size_t xrow = (size_t)H * 2 + 64;
  return (size_t)nstage * FSTAGE + (size_t)B * xrow + (2 * (size_t)nstage + 2) * 8 + sizeof(FPlan) +
         (size_t)E * 4 + 16;
}

struct FusedScratch {
  size_t rl, p13, p2, hf, cnt13, cnt2, gbar, status, total;
  int p13max, qmax, slots;
};

static size_t al2(size_t v) { return (v + 255) & ~size_t(255); }

// Scratch of the persistent path, always laid out for 8 tokens so that its position in the
// workspace and its counters do not depend on the call's batch; the counters, the grid barrier and
// the status word come first so that layers of either weight format sharing a workspace find the
// same (zero) words there.
FusedScratch fused_scratch(int H, int I_loc, int E, int B, int topk, int r_fmt) {
  (void)B;
  B = FMAXB;
  FusedScratch f{};
  const int T = I_loc / 16, NT = H / 16;
  const int P13s = (H / 32) / FCH, P13r = r_fmt == DSMOE_FMT_FP8 ? (H / 32) / FCH : (H / 64) / FCH;
  const int KC2s = I_loc / 32, KC2r = r_fmt == DSMOE_FMT_FP8 ? I_loc / 32 : I_loc / 64;
  const int P2s = (KC2s + FCH - 1) / FCH, P2r = (KC2r + FCH - 1) / FCH;
  const int P13max_any = (H / 32) / FCH;                       // FP8 parts bound both formats
  const int P2max_any = (I_loc / 32 + FCH - 1) / FCH;
  (void)P13s; (void)P13r; (void)P2s; (void)P2r;
  f.slots = B * topk + 1;
  f.p13max = P13max_any;
  f.qmax = B * topk * P2max_any + P2max_any;
  size_t o = 0;
  f.gbar = o; o += al2(8);
  f.status = o; o += al2(4);
  f.cnt2 = o; o += al2((size_t)NT * 4);
  f.cnt13 = o; o += al2((size_t)f.slots * T * 4);
  f.rl = o; o += al2((size_t)B * E * 4 * 8);
  f.p13 = o; o += al2((size_t)f.slots * T * f.p13max * 32 * 8 * 4);
  f.p2 = o; o += al2((size_t)NT * f.qmax * 32 * 4 * 4);
  f.hf = o; o += al2((size_t)f.slots * 8 * I_loc * 2);
  f.total = o;
  return f;
}

bool fused_supported(const dsmoe_layer_t* L, int B) {
  if (B < 1 || B > FMAXB || L->n_experts > FEMAX || L->hidden % 512 != 0 || L->hidden > FSTAGE) return false;
  int dev = 0, optin = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  return fused_smem_bytes(L->hidden, B, L->n_experts, 8) <= (size_t)optin;
}

int launch_fused(const dsmoe_layer_t* L, const void* x, int B, const uint8_t* image_mask, void* y, int y_dtype,
                 int64_t* idx, float* wt, float* scores, uint8_t* ws, cudaStream_t st) {
  int dev = 0, optin = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int nstage = 16;
  while (nstage > 8 && fused_smem_bytes(L->hidden, B, L->n_experts, nstage) > (size_t)optin) --nstage;
  const size_t smem = fused_smem_bytes(L->hidden, B, L->n_experts, nstage);
  DSMOE_REQUIRE(smem <= (size_t)optin, DSMOE_ERR_UNSUPPORTED, "fused: %zu bytes of shared memory needed", smem);
  const FusedScratch f = fused_scratch(L->hidden, L->inter_local, L->n_experts, B, L->topk, L->routed.fmt);

  FusedArgs a{};
  a.H = L->hidden;
  a.I_loc = L->inter_local;
  a.E = L->n_experts;
  a.B = B;
  a.topk = L->topk;
  a.score_func = L->score_func;
  a.route_scale = L->route_scale;
  a.wg = L->gate_w;
  a.bias = L->gate_bias;
  a.bias_vl = L->gate_bias_vl;
  a.image_mask = image_mask;
  a.x = (const __nv_bfloat16*)x;
  a.r_fmt = L->routed.fmt;
  a.r_w13 = L->routed.w13;
  a.r_w2 = L->routed.w2;
  a.r_w13_eb = L->routed.w13_expert_bytes;
  a.r_w2_eb = L->routed.w2_expert_bytes;
  a.s_w13 = L->shared.w13;
  a.s_w2 = L->shared.w2;
  a.y = y;
  a.y_f32 = y_dtype == DSMOE_DTYPE_F32;
  a.idx = idx;
  a.wt = wt;
  a.scores = scores;
  a.rl = (double*)(ws + f.rl);
  a.p13 = (float*)(ws + f.p13);
  a.p2 = (float*)(ws + f.p2);
  a.hf = (uint16_t*)(ws + f.hf);
  a.cnt13 = (unsigned*)(ws + f.cnt13);
  a.cnt2 = (unsigned*)(ws + f.cnt2);
  a.gbar = (unsigned*)(ws + f.gbar);
  a.status = (unsigned*)(ws + f.status);
  a.sh_idx = FMAXB * L->topk;
  a.nstage = nstage;
  a.xrow = L->hidden * 2 + 64;
  a.p13max = f.p13max;
  a.qmax = f.qmax;

  void (*kern)(FusedArgs) = L->routed.fmt == DSMOE_FMT_FP8 ? moe_fused_kernel<DSMOE_FMT_FP8> : moe_fused_kernel<DSMOE_FMT_FP4>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return cuda_status("fused: set smem");
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, FT, smem);
  DSMOE_REQUIRE(per_sm >= 1, DSMOE_ERR_UNSUPPORTED, "fused: kernel does not fit on an SM");
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(sms);
  cfg.blockDim = dim3(FT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
  if (e != cudaSuccess) {
    set_error("fused launch: %s", cudaGetErrorString(e));
    cudaGetLastError();
    return DSMOE_ERR_CUDA;
  }
  return DSMOE_OK;
}

}  // namespace dsmoe
