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
//   consumers  dequantize A fragments from the stage, mma.sync m16n8k16 (f16 x f16 -> fp32)
//              against the tokens' f16 fragments (shared memory), block scales on fp32 partials.
// Work distribution: every phase is a flat list of items (4-8.5 KB of packed chunks each); each
// CTA takes a contiguous span and each consumer warp a contiguous run of that span, so a warp
// accumulates the consecutive parts of a 16-row tile in registers and publishes one partial per
// tile it shares with other warps. The last contributor of a tile (counter in the workspace)
// re-derives the tile's segments from the same deterministic distribution and sums them in order,
// so results do not depend on timing.
// Phases:
//   R  router quarter-rows (fp64 accumulation) + the shared expert's w1|w3 parts (no routing
//      needed); a CTA arrives at grid barrier A when its router rows are done, and the shared-
//      expert work hides the barrier.
//   P  every CTA computes the same top-k and slot plan from the router partials.
//   1  routed w1|w3 parts; tile epilogue: clamp / SiLU / up / routing weight -> h (f16).
//   2  after grid barrier B: w2 parts (16 output rows x slot x 256 K); tile epilogue -> y.
// Every wait (mbarrier, grid barrier) is bounded by %globaltimer; on expiry the kernel records a
// status bit in the workspace, stops issuing work, lets its own copies land and returns.
#include "router.cuh"

namespace dsmoe {

constexpr int FW = 8;                  // consumer warps
constexpr int FT = (FW + 1) * 32;      // + producer warp
constexpr int FCH = 8;                 // packed chunks per w1|w3 item
constexpr int FSTAGE = FCH * 1088;     // bytes per ring stage (8 FP4 w1|w3 chunks, the largest item)
constexpr int FK2 = 256;               // K values per w2 item (8 FP8 chunks or 4 FP4 chunks)
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
  double* rl;        // [8][E][4] router quarter-row partial logits
  float* p13;        // [slots][T][p13max][32][8] w1|w3 tile-segment partials
  float* p2;         // [NT][qmax][32][4] w2 tile-segment partials (token columns)
  uint16_t* hf;      // [slots * 8][I_loc] h, f16, fragment order
  unsigned* cnt13;   // [slots][T]
  unsigned* cnt2;    // [NT]
  unsigned* gbar;    // [0] arrivals, [1] generation
  unsigned* status;  // [0]
  int sh_idx;        // scratch slot index of the shared expert
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
  int T, NT, KB, NR, NS, P13s, P13r, P2;
  int chunk13r, chunk2r, nch2r;
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
  g.P2 = (a.I_loc + FK2 - 1) / FK2;
  g.chunk13r = a.r_fmt == DSMOE_FMT_FP8 ? 1024 : 1088;
  g.chunk2r = a.r_fmt == DSMOE_FMT_FP8 ? 512 : 544;
  g.nch2r = a.r_fmt == DSMOE_FMT_FP8 ? FK2 / 32 : FK2 / 64;
  g.tile13r = w13_tile_bytes(a.r_fmt, a.H);
  g.tile13s = fp8_w13_tile_bytes(a.H);
  g.tile2r = w2_tile_bytes(a.r_fmt, a.I_loc);
  g.tile2s = fp8_w2_tile_bytes(a.I_loc);
  return g;
}

// ------------------------------------------------------------------ deterministic distribution
struct Span {
  int s, e;
};
__device__ __forceinline__ Span cta_span(int n, int c, int G) {
  return {(int)((long long)n * c / G), (int)((long long)n * (c + 1) / G)};
}
__device__ __forceinline__ Span warp_run(Span cs, int w) {
  const int nc = cs.e - cs.s, L = nc / FW, r = nc % FW;
  const int rs = cs.s + w * L + min(w, r);
  return {rs, rs + L + (w < r ? 1 : 0)};
}
// Calls f(first item of the segment - a) for every warp run that intersects [a, b), in order.
template <class F>
__device__ __forceinline__ void for_segments(int n, int G, int a, int b, F&& f) {
  int c = (int)(((long long)a * G) / n);
  while (c + 1 < G && cta_span(n, c + 1, G).s <= a) ++c;
  while (c > 0 && cta_span(n, c, G).s > a) --c;
  for (; c < G; ++c) {
    const Span cs = cta_span(n, c, G);
    if (cs.s >= b) break;
    for (int w = 0; w < FW; ++w) {
      const Span r = warp_run(cs, w);
      if (r.e <= a || r.s >= r.e) continue;
      if (r.s >= b) break;
      f(max(r.s, a) - a);
    }
  }
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

// ------------------------------------------------------------------ router
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

// ------------------------------------------------------------------ w1|w3
// One item (8 chunks of a 16-row tile, part p) accumulated into acc1 / acc3.
template <int FMT>
__device__ __forceinline__ void w13_accum(const FusedArgs& a, const Geo& G, const uint8_t* stage, const uint8_t* xrow,
                                          const uint8_t* tile_g, int p, int lane, float (&acc1)[4], float (&acc3)[4]) {
  const int g = lane >> 2, tq = lane & 3;
  float t1[4] = {0.f, 0.f, 0.f, 0.f}, t3[4] = {0.f, 0.f, 0.f, 0.f};
  if (FMT == DSMOE_FMT_FP8) {
    const float* sc = reinterpret_cast<const float*>(tile_g + (long long)(a.H / 32) * 1024);
    const float s1a = __ldg(sc + 2 * p), s1b = __ldg(sc + 2 * p + 1);
    const float s3a = __ldg(sc + G.KB + 2 * p), s3b = __ldg(sc + G.KB + 2 * p + 1);
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
      if (c == 3) {
        fma4s(acc1, t1, s1a);
        fma4s(acc3, t3, s3a);
      } else if (c == 7) {
        fma4s(acc1, t1, s1b);
        fma4s(acc3, t3, s3b);
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
}

// Tile epilogue: clamp, SiLU(gate) * up * routing weight -> h (f16, w2's fragment order).
__device__ __forceinline__ void w13_epilogue(const FusedArgs& a, const FPlan& pl, int sidx, int t, const float (&s)[8],
                                             int ntok, const int* toks, const float* wts, int lane) {
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

// A warp's contribution to one tile ends: publish it, or finish the tile if it is complete.
// [a0, a0 + P) are the tile's items in the phase (n items); the warp covered seg_np of them from seg_first.
__device__ void w13_flush(const FusedArgs& a, const Geo& G, const FPlan& pl, int n, int a0, int P, int seg_first,
                          int seg_np, int sidx, int t, const float (&acc1)[4], const float (&acc3)[4], int ntok,
                          const int* toks, const float* wts, int lane) {
  float s[8] = {acc1[0], acc1[1], acc1[2], acc1[3], acc3[0], acc3[1], acc3[2], acc3[3]};
  if (seg_np == P) {
    w13_epilogue(a, pl, sidx, t, s, ntok, toks, wts, lane);
    return;
  }
  float* base = a.p13 + (((long long)sidx * G.T + t) * a.p13max) * 32 * 8;
  float* dst = base + ((long long)(seg_first - a0) * 32 + lane) * 8;
  *reinterpret_cast<float4*>(dst) = make_float4(s[0], s[1], s[2], s[3]);
  *reinterpret_cast<float4*>(dst + 4) = make_float4(s[4], s[5], s[6], s[7]);
  __threadfence();
  __syncwarp();
  unsigned old = 0;
  if (lane == 0) old = atomicAdd(a.cnt13 + sidx * G.T + t, (unsigned)seg_np);
  old = __shfl_sync(0xffffffffu, old, 0);
  if ((int)old + seg_np != P) return;
  __threadfence();
#pragma unroll
  for (int j = 0; j < 8; ++j) s[j] = 0.f;
  for_segments(n, gridDim.x, a0, a0 + P, [&](int q) {
    const float* src = base + ((long long)q * 32 + lane) * 8;
    const uint4 v0 = ld_cg16(src), v1 = ld_cg16(src + 4);
    s[0] += __uint_as_float(v0.x); s[1] += __uint_as_float(v0.y);
    s[2] += __uint_as_float(v0.z); s[3] += __uint_as_float(v0.w);
    s[4] += __uint_as_float(v1.x); s[5] += __uint_as_float(v1.y);
    s[6] += __uint_as_float(v1.z); s[7] += __uint_as_float(v1.w);
  });
  w13_epilogue(a, pl, sidx, t, s, ntok, toks, wts, lane);
  if (lane == 0) a.cnt13[sidx * G.T + t] = 0u;
}

// ------------------------------------------------------------------ w2
// The 8 k32 blocks of h this lane feeds to one w2 item (slot row sidx*8+g, K range p*256..).
__device__ __forceinline__ void load_h(const FusedArgs& a, int sidx, int p, int lane, uint4 (&hb)[8]) {
  const int g = lane >> 2, tq = lane & 3;
  const int kc = a.I_loc / 32;
  const uint8_t* hrow = reinterpret_cast<const uint8_t*>(a.hf + (long long)(sidx * 8 + g) * a.I_loc) + tq * 16;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (p * 8 + i < kc) hb[i] = ld_cg16(hrow + (long long)(p * 8 + i) * 64);
}

// One w2 item of slot s accumulated into out[] (token columns: rows g, g+8 x tokens 2tq, 2tq+1).
template <int FMT>
__device__ __forceinline__ void w2_accum(const FusedArgs& a, const FPlan& pl, const uint8_t* stage, const uint8_t* tile_g,
                                         int s, int p, const uint4 (&hb)[8], int lane, float (&out)[4]) {
  const int g = lane >> 2, tq = lane & 3;
  float acc[4] = {0.f, 0.f, 0.f, 0.f}, tt[4] = {0.f, 0.f, 0.f, 0.f};
  if (FMT == DSMOE_FMT_FP8) {
    const int KC = a.I_loc / 32;
    const float* sc = reinterpret_cast<const float*>(tile_g + (long long)KC * 512);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (p * 8 + i < KC) {
        const uint4 A0 = lds16(stage + i * 512 + lane * 16);
        uint32_t A[4];
        a_frag_fp8(A, A0.x, A0.y); mma16816(tt, A, hb[i].x, hb[i].y);
        a_frag_fp8(A, A0.z, A0.w); mma16816(tt, A, hb[i].z, hb[i].w);
        fma4s(acc, tt, __ldg(sc + p * 8 + i));
      }
    }
  } else {
    const int KC = a.I_loc / 64;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (p * 4 + i < KC) {
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
  // slot columns -> token columns
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int tok = 2 * tq + h;
    const int col = tok < a.B ? pl.col_of[s][tok] : -1;
    const int src = g * 4 + (col < 0 ? 0 : col >> 1);
    const float v0 = __shfl_sync(0xffffffffu, acc[0], src), v1 = __shfl_sync(0xffffffffu, acc[1], src);
    const float v2 = __shfl_sync(0xffffffffu, acc[2], src), v3 = __shfl_sync(0xffffffffu, acc[3], src);
    if (col >= 0) {
      out[h] += (col & 1) ? v1 : v0;
      out[2 + h] += (col & 1) ? v3 : v2;
    }
  }
}

__device__ __forceinline__ void w2_epilogue(const FusedArgs& a, int nt, const float (&s)[4], int lane) {
  const int g = lane >> 2, tq = lane & 3;
#pragma unroll
  for (int q4 = 0; q4 < 4; ++q4) {
    const int row = nt * 16 + (q4 >= 2 ? g + 8 : g), tok = 2 * tq + (q4 & 1);
    if (tok < a.B) {
      const long long o = (long long)tok * a.H + row;
      if (a.y_f32)
        reinterpret_cast<float*>(a.y)[o] = s[q4];
      else
        reinterpret_cast<__nv_bfloat16*>(a.y)[o] = __float2bfloat16_rn(s[q4]);
    }
  }
}

__device__ void w2_flush(const FusedArgs& a, int n, int Q, int nt, int seg_first, int seg_np, const float (&out)[4],
                         int lane) {
  float s[4] = {out[0], out[1], out[2], out[3]};
  const int a0 = nt * Q;
  if (seg_np == Q) {
    w2_epilogue(a, nt, s, lane);
    return;
  }
  float* base = a.p2 + ((long long)nt * a.qmax) * 32 * 4;
  *reinterpret_cast<float4*>(base + ((long long)(seg_first - a0) * 32 + lane) * 4) = make_float4(s[0], s[1], s[2], s[3]);
  __threadfence();
  __syncwarp();
  unsigned old = 0;
  if (lane == 0) old = atomicAdd(a.cnt2 + nt, (unsigned)seg_np);
  old = __shfl_sync(0xffffffffu, old, 0);
  if ((int)old + seg_np != Q) return;
  __threadfence();
  s[0] = s[1] = s[2] = s[3] = 0.f;
  for_segments(n, gridDim.x, a0, a0 + Q, [&](int q) {
    const uint4 v = ld_cg16(base + ((long long)q * 32 + lane) * 4);
    s[0] += __uint_as_float(v.x); s[1] += __uint_as_float(v.y);
    s[2] += __uint_as_float(v.z); s[3] += __uint_as_float(v.w);
  });
  w2_epilogue(a, nt, s, lane);
  if (lane == 0) a.cnt2[nt] = 0u;
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
  const Span spanR = cta_span(nR, cta, G);
  const int my_router = max(0, min(spanR.e, geo.NR) - spanR.s);

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
    // items of a CTA span in the consumers' order: the k-th item of every warp run, warp by warp
    auto issue_span = [&](Span cs, auto&& item) {
      const int L = (cs.e - cs.s + FW - 1) / FW;
      for (int k = 0; k < L && ok; ++k)
        for (int w = 0; w < FW && ok; ++w) {
          const Span r = warp_run(cs, w);
          if (r.s + k < r.e) item(r.s + k);
        }
    };
    issue_span(spanR, [&](int i) {
      if (i < geo.NR) {
        issue(a.wg + (long long)(i >> 2) * a.H + (i & 3) * (a.H / 4), (uint32_t)a.H);
      } else {
        const int i2 = i - geo.NR, t = i2 / geo.P13s, p = i2 % geo.P13s;
        issue(a.s_w13 + t * geo.tile13s + (long long)p * FCH * 1024, FCH * 1024);
      }
    });
    if (ok && !mbar_wait(planbar, 0, 4 * kWaitNs)) {
      atomicOr(a.status, ST_PLAN);
      ok = false;
    }
    if (ok) {
      const int nr = pl.n_routed;
      const int N1 = nr * geo.T * geo.P13r;
      issue_span(cta_span(N1, cta, G), [&](int i) {
        const int tile = i / geo.P13r, p = i % geo.P13r, s = tile / geo.T, t = tile % geo.T;
        const uint8_t* base = a.r_w13 + (long long)pl.expert[s] * a.r_w13_eb + t * geo.tile13r;
        issue(base + (long long)p * FCH * geo.chunk13r, (uint32_t)(FCH * geo.chunk13r));
      });
      const int Q = (nr + 1) * geo.P2;
      const int N2 = geo.NT * Q;
      issue_span(cta_span(N2, cta, G), [&](int i) {
        const int nt = i / Q, jq = i % Q, s = jq / geo.P2, p = jq % geo.P2;
        if (s < nr) {
          const int kc = a.I_loc / (RFMT == DSMOE_FMT_FP8 ? 32 : 64);
          const int nch = min(geo.nch2r, kc - p * geo.nch2r);
          issue(a.r_w2 + (long long)pl.expert[s] * a.r_w2_eb + nt * geo.tile2r + (long long)p * geo.nch2r * geo.chunk2r,
                (uint32_t)(nch * geo.chunk2r));
        } else {
          const int nch = min(8, a.I_loc / 32 - p * 8);
          issue(a.s_w2 + nt * geo.tile2s + (long long)p * 8 * 512, (uint32_t)(nch * 512));
        }
      });
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
      p = e2 - 15;  // m * 2^-p in [2^14, 2^15): inside f16 range with room to spare
    }
    if (lane == 0) pl.xscale[warp] = ldexpf(1.0f, p);
    const float inv = ldexpf(1.0f, -p);
    for (int c = lane; c < a.H / 32; c += 32) {
      float v[32];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(xr + 32 * c + 8 * q));
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          v[8 * q + 2 * h] = __uint_as_float(w[h] << 16) * inv;
          v[8 * q + 2 * h + 1] = __uint_as_float(w[h] & 0xFFFF0000u) * inv;
        }
      }
#pragma unroll
      for (int tq = 0; tq < 4; ++tq)
        *reinterpret_cast<uint4*>(xf + (long long)warp * a.xrow + c * 64 + tq * 16) =
            make_uint4(pack_f16x2(v[2 * tq], v[2 * tq + 1]), pack_f16x2(v[2 * tq + 8], v[2 * tq + 9]),
                       pack_f16x2(v[2 * tq + 16], v[2 * tq + 17]), pack_f16x2(v[2 * tq + 24], v[2 * tq + 25]));
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

  int jbase = 0;  // sequence number of the phase's first item in this CTA (the producer's order)

  // ---- phase R: router quarter-rows, then the shared expert's w1|w3 parts
  {
    const Span run = warp_run(spanR, warp);
    int cur = -1, seg_first = 0, seg_np = 0, n_router = 0;
    float acc1[4] = {0.f, 0.f, 0.f, 0.f}, acc3[4] = {0.f, 0.f, 0.f, 0.f};
    const uint8_t* xrow = xf + (long long)shared_toks[min(lane >> 2, a.B - 1)] * a.xrow;
    for (int i = run.s; i < run.e; ++i) {
      const int jj = jbase + 8 * (i - run.s) + warp;
      if (!wait_full(jj)) break;
      const uint8_t* stage = ring + (size_t)(jj % a.nstage) * FSTAGE;
      if (i < geo.NR) {
        router_item(a, stage, i >> 2, i & 3, lane);
        ++n_router;
      } else {
        const int i2 = i - geo.NR, t = i2 / geo.P13s, p = i2 % geo.P13s;
        if (t != cur) {
          if (cur >= 0)
            w13_flush(a, geo, pl, nR, geo.NR + cur * geo.P13s, geo.P13s, seg_first, seg_np, a.sh_idx, cur, acc1, acc3,
                      a.B, shared_toks, shared_wts, lane);
          cur = t;
          seg_first = i;
          seg_np = 0;
#pragma unroll
          for (int q = 0; q < 4; ++q) acc1[q] = acc3[q] = 0.f;
        }
        w13_accum<DSMOE_FMT_FP8>(a, geo, stage, xrow, a.s_w13 + t * geo.tile13s, p, lane, acc1, acc3);
        ++seg_np;
      }
      release(jj);
      if (i + 1 == min(run.e, geo.NR)) {  // this warp's last router row: count its rows toward barrier A
        __threadfence();
        __syncwarp();
        if (lane == 0) {
          const unsigned done = atomicAdd(&pl.router_done, (unsigned)n_router) + n_router;
          if ((int)done == my_router) pl.gen_a = grid_arrive(a.gbar, G);
        }
      }
    }
    if (cur >= 0 && !pl.abort)
      w13_flush(a, geo, pl, nR, geo.NR + cur * geo.P13s, geo.P13s, seg_first, seg_np, a.sh_idx, cur, acc1, acc3, a.B,
                shared_toks, shared_wts, lane);
  }
  jbase += spanR.e - spanR.s;
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
  __threadfence();

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
  {
    const Span span = cta_span(N1, cta, G);
    const Span run = warp_run(span, warp);
    int cur = -1, seg_first = 0, seg_np = 0;
    float acc1[4] = {0.f, 0.f, 0.f, 0.f}, acc3[4] = {0.f, 0.f, 0.f, 0.f};
    for (int i = run.s; i < run.e; ++i) {
      const int jj = jbase + 8 * (i - run.s) + warp;
      if (!wait_full(jj)) break;
      const uint8_t* stage = ring + (size_t)(jj % a.nstage) * FSTAGE;
      const int tile = i / geo.P13r, p = i % geo.P13r, s = tile / geo.T, t = tile % geo.T;
      if (tile != cur) {
        if (cur >= 0) {
          const int cs = cur / geo.T;
          w13_flush(a, geo, pl, N1, cur * geo.P13r, geo.P13r, seg_first, seg_np, cs, cur % geo.T, acc1, acc3,
                    pl.ntok[cs], pl.tok[cs], pl.wt[cs], lane);
        }
        cur = tile;
        seg_first = i;
        seg_np = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) acc1[q] = acc3[q] = 0.f;
      }
      const uint8_t* xrow = xf + (long long)pl.tok[s][min(lane >> 2, pl.ntok[s] - 1)] * a.xrow;
      const uint8_t* tile_g = a.r_w13 + (long long)pl.expert[s] * a.r_w13_eb + t * geo.tile13r;
      w13_accum<RFMT>(a, geo, stage, xrow, tile_g, p, lane, acc1, acc3);
      ++seg_np;
      release(jj);
    }
    if (cur >= 0 && !pl.abort) {
      const int cs = cur / geo.T;
      w13_flush(a, geo, pl, N1, cur * geo.P13r, geo.P13r, seg_first, seg_np, cs, cur % geo.T, acc1, acc3, pl.ntok[cs],
                pl.tok[cs], pl.wt[cs], lane);
    }
    jbase += span.e - span.s;
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
  __threadfence();

  // ---- phase 2: w2 (h operands double-buffered in registers)
  {
    const int Q = (nr + 1) * geo.P2;
    const int N2 = geo.NT * Q;
    const Span span = cta_span(N2, cta, G);
    const Span run = warp_run(span, warp);
    int cur = -1, seg_first = 0, seg_np = 0;
    float out[4] = {0.f, 0.f, 0.f, 0.f};
    uint4 hA[8], hB[8];
    auto step = [&](int i, const uint4(&hb)[8]) -> bool {
      const int jj = jbase + 8 * (i - run.s) + warp;
      if (!wait_full(jj)) return false;
      const uint8_t* stage = ring + (size_t)(jj % a.nstage) * FSTAGE;
      const int nt = i / Q, jq = i % Q, s = jq / geo.P2, p = jq % geo.P2;
      if (nt != cur) {
        if (cur >= 0) w2_flush(a, N2, Q, cur, seg_first, seg_np, out, lane);
        cur = nt;
        seg_first = i;
        seg_np = 0;
        out[0] = out[1] = out[2] = out[3] = 0.f;
      }
      if (s < nr)
        w2_accum<RFMT>(a, pl, stage, a.r_w2 + (long long)pl.expert[s] * a.r_w2_eb + nt * geo.tile2r, s, p, hb, lane, out);
      else
        w2_accum<DSMOE_FMT_FP8>(a, pl, stage, a.s_w2 + nt * geo.tile2s, s, p, hb, lane, out);
      ++seg_np;
      release(jj);
      return true;
    };
    auto fetch = [&](int i, uint4(&hb)[8]) {
      const int jq = i % Q, s = jq / geo.P2;
      load_h(a, s < nr ? s : a.sh_idx, jq % geo.P2, lane, hb);
    };
    if (run.s < run.e) fetch(run.s, hA);
    for (int i = run.s; i < run.e; i += 2) {
      if (i + 1 < run.e) fetch(i + 1, hB);
      if (!step(i, hA)) break;
      if (i + 1 < run.e) {
        if (i + 2 < run.e) fetch(i + 2, hA);
        if (!step(i + 1, hB)) break;
      }
    }
    if (cur >= 0 && !pl.abort) w2_flush(a, N2, Q, cur, seg_first, seg_np, out, lane);
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
  (void)r_fmt;
  B = FMAXB;
  FusedScratch f{};
  const int T = I_loc / 16, NT = H / 16;
  f.slots = B * topk + 1;
  f.p13max = (H / 32) / FCH;                        // FP8 parts per tile bound both formats
  f.qmax = f.slots * ((I_loc + FK2 - 1) / FK2);     // w2 items per 16 output rows
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

// Per-device constants, looked up once (attribute queries cost microseconds per call).
struct DevInfo {
  int sms = 0, optin = 0;
  bool attr_set[2] = {false, false};
};
static DevInfo g_dev[64];

static DevInfo& dev_info() {
  int dev = 0;
  cudaGetDevice(&dev);
  DevInfo& d = g_dev[dev & 63];
  if (d.sms == 0) {
    cudaDeviceGetAttribute(&d.optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
  }
  return d;
}

bool fused_supported(const dsmoe_layer_t* L, int B) {
  if (B < 1 || B > FMAXB || L->n_experts > FEMAX || L->hidden % 512 != 0 || L->hidden > FSTAGE) return false;
  return fused_smem_bytes(L->hidden, B, L->n_experts, 8) <= (size_t)dev_info().optin;
}

int launch_fused(const dsmoe_layer_t* L, const void* x, int B, const uint8_t* image_mask, void* y, int y_dtype,
                 int64_t* idx, float* wt, float* scores, uint8_t* ws, cudaStream_t st, void* const* events) {
  DevInfo& d = dev_info();
  const int optin = d.optin, sms = d.sms;
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

  const int fi = L->routed.fmt == DSMOE_FMT_FP8 ? 0 : 1;
  void (*kern)(FusedArgs) = fi == 0 ? moe_fused_kernel<DSMOE_FMT_FP8> : moe_fused_kernel<DSMOE_FMT_FP4>;
  if (!d.attr_set[fi]) {
    // the largest dynamic shared memory any call can ask for; set once per device and format
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, optin) != cudaSuccess)
      return cuda_status("fused: set smem");
    d.attr_set[fi] = true;
  }
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
  if (events) {
    cudaEventRecord((cudaEvent_t)events[0], st);
    cudaEventRecord((cudaEvent_t)events[1], st);
    cudaEventRecord((cudaEvent_t)events[2], st);
  }
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
  if (events) cudaEventRecord((cudaEvent_t)events[3], st);
  if (e != cudaSuccess) {
    set_error("fused launch: %s", cudaGetErrorString(e));
    cudaGetLastError();
    return DSMOE_ERR_CUDA;
  }
  return DSMOE_OK;
}

}  // namespace dsmoe
