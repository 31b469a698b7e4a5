// One persistent kernel per MoE layer for decode batches of 1..8 tokens.
//
// Replaces the per-layer sequence of the reference's decode -- device router GEMV, host top-k,
// host->device control write, SlotCat gather, w1/w3/shared matmuls, Q20 SwiGLU, w2 matmuls
// (dsv41/tt/model.py:400-442; dsv41/tt/moe.py:108-180; dsv41/kernels/slot_cat.cpp) -- with one
// launch that streams every weight byte the step needs exactly once.
//
// Shape: one CTA per SM (cooperative launch), 7 consumer warps + 1 producer warp.
//   producer   one thread issues 1-D bulk copies (cp.async.bulk, the TMA engine) of everything a
//              work item reads -- its packed weights, their FP8 scales and, for w2 items, the h
//              rows of its slot -- into a ring of 14 x 8.5 KB shared-memory stages, counted
//              on one mbarrier per stage. It runs ahead across phase boundaries: w2 weights stream
//              in while the grid still waits for the last w1|w3 tiles; their h rows follow as soon
//              as grid barrier B has passed.
//   consumers  read nothing from global memory on the streaming path: A fragments straight from
//              the stage (FP8 bytes as they are, FP4 expanded to e4m3 with integer operations),
//              mma.sync m16n8k32 e4m3 x e4m3 -> fp32 against the tokens' e4m3 hi / lo rows (shared
//              memory) or the stage's h rows, block scales on the fp32 partials.
// Work distribution: every phase is a flat list of items (2-8.5 KB each); each CTA takes a
// contiguous span and each consumer warp a contiguous run of it, so a warp accumulates the
// consecutive parts of a 16-row tile in registers and publishes one partial per tile it shares.
// The last contributor of a tile (counter in the workspace) re-derives the tile's segments from
// the same deterministic distribution and sums them in order: results do not depend on timing.
// Phases:
//   R  router quarter-rows (fp64) and the shared expert's w1|w3 parts (no routing needed), both
//      spread over all CTAs; a CTA arrives at grid barrier A when its router rows are done.
//   P  every CTA computes the same scores, top-k and slot plan (shared memory scratch).
//   1  routed w1|w3 parts; tile epilogue: clamp / SiLU / up -> h (e4m3 hi / lo rows).
//   2  after grid barrier B: w2 parts (16 output rows x slot x 256 K), routing weight on the fp32
//      partials; tile epilogue -> y.
// Every wait (mbarrier, grid barrier) is bounded by %globaltimer; on expiry the kernel records a
// status bit in the workspace, stops issuing work, lets its own copies land and returns.
#include "router.cuh"

namespace dsmoe {

constexpr int FW = 7;                  // consumer warps (+1 producer: two warps per SM sub-partition)
constexpr int FT = (FW + 1) * 32;      // + producer warp
constexpr int FCH = 8;                 // packed chunks per w1|w3 item
constexpr int FSTAGE = FCH * 1088;     // bytes per ring stage (8 FP4 w1|w3 chunks, the largest item)
constexpr int FK2 = 256;               // K values per w2 item (8 FP8 chunks or 4 FP4 chunks)
constexpr int FH2 = kFp8W2Item;        // w2 stage: the packed item (<= 4128 B), then the slot's h
constexpr int FH2T = 8 * kHPartK + 64; // rows: hi rows at FH2, lo rows FH2T further (the 64-byte
                                       // offset puts the two terms in opposite bank halves)
static_assert(FH2 + FH2T + 8 * kHPartK <= FSTAGE, "w2 stage overflow");
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
  uint8_t* hq;       // [slots] h rows, e4m3 hi / lo (hq_off)
  unsigned* cnt13;   // [slots][T]
  unsigned* cnt2;    // [NT]
  unsigned* gbar;    // [0] arrivals, [1] generation
  unsigned* status;  // [0]
  int sh_idx;        // scratch slot index of the shared expert
  int nstage, xrs, p13max, qmax;   // xrs: bytes per token row (hi or lo) in shared memory
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
// Phases 1 and 2: item i of n belongs to CTA span / warp run as above. Calls f(first item of the
// segment - a) for every warp run that intersects [a, b), in order.
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
// Phase R: CTA c's local list is its router span (over NR) followed by its shared-expert span
// (over NS); warp runs split the local list. Same contract as for_segments, over the NS items.
template <class F>
__device__ __forceinline__ void for_segments_R(int NR, int NS, int G, int a, int b, F&& f) {
  int c = (int)(((long long)a * G) / NS);
  while (c + 1 < G && cta_span(NS, c + 1, G).s <= a) ++c;
  while (c > 0 && cta_span(NS, c, G).s > a) --c;
  for (; c < G; ++c) {
    const Span ss = cta_span(NS, c, G);
    if (ss.s >= b) break;
    const Span rs = cta_span(NR, c, G);
    const int rc = rs.e - rs.s;
    const Span local = {0, rc + ss.e - ss.s};
    for (int w = 0; w < FW; ++w) {
      const Span r = warp_run(local, w);
      const int s0 = max(r.s, rc) - rc + ss.s, s1 = r.e - rc + ss.s;  // the run's shared items
      if (r.e <= rc || s1 <= a || s0 >= s1) continue;
      if (s0 >= b) break;
      f(max(s0, a) - a);
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
__device__ __forceinline__ float ldsf(const uint8_t* p) { return *reinterpret_cast<const float*>(p); }

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }

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
    __nanosleep(32);
  }
  return true;
}

// ------------------------------------------------------------------ router
// Router quarter-row: 1/4 of gate_w[r] (H/4 fp32, in the stage) . x[b] for every token, fp64.
// The token's values come from global memory (L1-resident after the first row); each token's
// loads are all issued before its multiply-adds.
__device__ void router_item(const FusedArgs& a, const uint8_t* stage, int r, int q, int lane) {
  const float4* wv = reinterpret_cast<const float4*>(stage);
  const int n4 = a.H / 16;  // float4 per quarter (<= 512 for H <= 8192)
  for (int b = 0; b < a.B; ++b) {
    const __nv_bfloat16* xr = a.x + (long long)b * a.H + q * (a.H / 4);
    uint2 xv[16];
#pragma unroll
    for (int it = 0; it < 16; ++it) {
      const int f = lane + 32 * it;
      if (f < n4) xv[it] = __ldg(reinterpret_cast<const uint2*>(xr + 4 * f));
    }
    double acc = 0.0;
#pragma unroll
    for (int it = 0; it < 16; ++it) {
      const int f = lane + 32 * it;
      if (f < n4) {
        const float4 w = wv[f];
        acc = fma((double)__uint_as_float(xv[it].x << 16), (double)w.x, acc);
        acc = fma((double)__uint_as_float(xv[it].x & 0xFFFF0000u), (double)w.y, acc);
        acc = fma((double)__uint_as_float(xv[it].y << 16), (double)w.z, acc);
        acc = fma((double)__uint_as_float(xv[it].y & 0xFFFF0000u), (double)w.w, acc);
      }
    }
    acc = warp_sum_d(acc);
    if (lane == 0) a.rl[((long long)b * a.E + r) * 4 + q] = acc;
  }
}

// ------------------------------------------------------------------ w1|w3
// One item (8 chunks of a 16-row tile, part p) accumulated into acc1 / acc3 for NTL n-tiles of
// slot tokens: C columns 2u, 2u + 1 of n-tile j hold the hi and lo terms of slot token 4j + u.
// xr[j] is the lane's token row in shared memory (B column g of n-tile j). Scales come with the
// weights (FP8: 16 bytes after the 8 chunks; FP4: inside each chunk).
template <int FMT, int NTL>
__device__ __forceinline__ void w13_accum(const uint8_t* stage, const uint8_t* const* xr, int p, int lane,
                                          float (&acc1)[2][4], float (&acc3)[2][4]) {
  const int g = lane >> 2;
  if (FMT == DSMOE_FMT_FP8) {
#pragma unroll
    for (int blk = 0; blk < 2; ++blk) {  // two 128-K blocks, four chunks each, one MMA chain per
      uint4 X[NTL][2];                   // matrix and n-tile (seven warps hide its latency)
#pragma unroll
      for (int j = 0; j < NTL; ++j) {
        X[j][0] = lds16(xr[j] + (4 * p + 2 * blk) * 64);
        X[j][1] = lds16(xr[j] + (4 * p + 2 * blk + 1) * 64);
      }
      float u1[NTL][4], u3[NTL][4];
#pragma unroll
      for (int j = 0; j < NTL; ++j)
#pragma unroll
        for (int q = 0; q < 4; ++q) u1[j][q] = u3[j][q] = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 A1 = lds16(stage + (4 * blk + c) * 1024 + lane * 16);
        const uint4 A3 = lds16(stage + (4 * blk + c) * 1024 + 512 + lane * 16);
#pragma unroll
        for (int j = 0; j < NTL; ++j) {
          const uint4 xb = X[j][c >> 1];
          const uint32_t b0 = (c & 1) ? xb.z : xb.x, b1 = (c & 1) ? xb.w : xb.y;
          mma_e4m3(u1[j], A1.x, A1.y, A1.z, A1.w, b0, b1);
          mma_e4m3(u3[j], A3.x, A3.y, A3.z, A3.w, b0, b1);
        }
      }
      const float s1 = ldsf(stage + FCH * 1024 + 4 * fp8_w13_scale_index(blk, 0));
      const float s3 = ldsf(stage + FCH * 1024 + 4 * fp8_w13_scale_index(blk, 1));
#pragma unroll
      for (int j = 0; j < NTL; ++j)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          acc1[j][q] = fmaf(u1[j][q], s1, acc1[j][q]);
          acc3[j][q] = fmaf(u3[j][q], s3, acc3[j][q]);
        }
    }
  } else {
#pragma unroll
    for (int c0 = 0; c0 < FCH; c0 += 2) {  // two chunks (four k32 MMAs per matrix and n-tile) at a time
      uint4 A1[2], A3[2], X[2][NTL];
      uint32_t S1[2], S3[2];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const uint8_t* ch = stage + (c0 + c) * 1088;
        A1[c] = lds16(ch + lane * 16);
        A3[c] = lds16(ch + 512 + lane * 16);
        S1[c] = lds32(ch + 1024 + 4 * g);
        S3[c] = lds32(ch + 1056 + 4 * g);
#pragma unroll
        for (int j = 0; j < NTL; ++j) X[c][j] = lds16(xr[j] + (FCH * p + c0 + c) * 64);
      }
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        fp4_chunk_mma<NTL>(A1[c], S1[c], X[c], acc1);
        fp4_chunk_mma<NTL>(A3[c], S3[c], X[c], acc3);
      }
    }
  }
}

// Tile epilogue. v[4j + 0..3] = gate row g, gate row g + 8, up row g, up row g + 8 of slot token
// 4j + tq, before the token's pre-scale and the weight-format factor fmtf. Clamp, SiLU(gate) * up
// -> h, written as e4m3 hi / lo bytes (times kHScale) where w2 reads them.
__device__ __forceinline__ void w13_epilogue(const FusedArgs& a, const FPlan& pl, int sidx, int t, const float (&v)[8],
                                             int ntok, const int* toks, float fmtf, int lane) {
  const int g = lane >> 2, tq = lane & 3;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int q = 4 * j + tq;
    if (q < ntok) {
      const float f = pl.xscale[toks[q]] * fmtf;
      float h[2];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const float gv = fminf(v[4 * j + r] * f, 10.0f);
        const float uv = fminf(fmaxf(v[4 * j + 2 + r] * f, -10.0f), 10.0f);
        h[r] = silu_f(gv) * uv * kHScale;
      }
      uint32_t hi2, lo2;
      split2_e4m3(h[0], h[1], hi2, lo2);
      const int k = 16 * t + g;
      a.hq[hq_off(a.I_loc, sidx, q, 0, k)] = (uint8_t)hi2;
      a.hq[hq_off(a.I_loc, sidx, q, 0, k + 8)] = (uint8_t)(hi2 >> 8);
      a.hq[hq_off(a.I_loc, sidx, q, 1, k)] = (uint8_t)lo2;
      a.hq[hq_off(a.I_loc, sidx, q, 1, k + 8)] = (uint8_t)(lo2 >> 8);
    }
  }
}

// A warp's contribution to one tile ends: publish it, or finish the tile if the warp covered all
// of it. seg_rel = the segment's first item minus the tile's first item. `segs` enumerates the
// tile's segments (same order everywhere) for the last contributor.
template <class Segs>
__device__ void w13_flush(const FusedArgs& a, const Geo& G, const FPlan& pl, int P, int seg_rel, int seg_np, int sidx,
                          int t, const float (&acc1)[2][4], const float (&acc3)[2][4], int ntok, const int* toks,
                          float fmtf, int lane, Segs&& segs) {
  float s[8];
#pragma unroll
  for (int j = 0; j < 2; ++j) {  // hi + lo / 16 per row
    s[4 * j] = acc1[j][0] + acc1[j][1] * kLoInv;
    s[4 * j + 1] = acc1[j][2] + acc1[j][3] * kLoInv;
    s[4 * j + 2] = acc3[j][0] + acc3[j][1] * kLoInv;
    s[4 * j + 3] = acc3[j][2] + acc3[j][3] * kLoInv;
  }
  if (seg_np == P) {
    w13_epilogue(a, pl, sidx, t, s, ntok, toks, fmtf, lane);
    return;
  }
  float* base = a.p13 + (((long long)sidx * G.T + t) * a.p13max) * 32 * 8;
  float* dst = base + ((long long)seg_rel * 32 + lane) * 8;
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
  segs([&](int q) {
    const float* src = base + ((long long)q * 32 + lane) * 8;
    const uint4 v0 = ld_cg16(src), v1 = ld_cg16(src + 4);
    s[0] += __uint_as_float(v0.x); s[1] += __uint_as_float(v0.y);
    s[2] += __uint_as_float(v0.z); s[3] += __uint_as_float(v0.w);
    s[4] += __uint_as_float(v1.x); s[5] += __uint_as_float(v1.y);
    s[6] += __uint_as_float(v1.z); s[7] += __uint_as_float(v1.w);
  });
  w13_epilogue(a, pl, sidx, t, s, ntok, toks, fmtf, lane);
  if (lane == 0) a.cnt13[sidx * G.T + t] = 0u;
}

// ------------------------------------------------------------------ w2
// One w2 item of slot s (weights, FP8 scales and the slot's h rows all in the stage) accumulated
// into out[] in token columns: rows g, g+8 x tokens 2tq, 2tq+1, with the routing weight.
template <int FMT, int NTL>
__device__ __forceinline__ void w2_accum(const FusedArgs& a, const FPlan& pl, const uint8_t* stage, int s, int p,
                                         int lane, float (&out)[4]) {
  const int g = lane >> 2, tq = lane & 3;
  const int ntok = pl.ntok[s];
  const uint8_t* hr[NTL];
#pragma unroll
  for (int j = 0; j < NTL; ++j) hr[j] = stage + FH2 + (g & 1) * FH2T + min(4 * j + (g >> 1), ntok - 1) * kHPartK + tq * 16;
  float tot[NTL][4];
#pragma unroll
  for (int j = 0; j < NTL; ++j)
#pragma unroll
    for (int q = 0; q < 4; ++q) tot[j][q] = 0.f;
  if (FMT == DSMOE_FMT_FP8) {
    const int nch = min(8, a.I_loc / 32 - p * 8);
    const uint8_t* sc = stage + nch * 512;
#pragma unroll
    for (int b = 0; b < 4; ++b) {  // 64-K blocks: two chunks each
      if (2 * b < nch) {
        uint4 Hb[NTL];
#pragma unroll
        for (int j = 0; j < NTL; ++j) Hb[j] = lds16(hr[j] + b * 64);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int i = 2 * b + h;
          if (i < nch) {
            const uint4 A0 = lds16(stage + i * 512 + lane * 16);
            const float si = ldsf(sc + 4 * i);
#pragma unroll
            for (int j = 0; j < NTL; ++j) {
              float d[4];
              mma_e4m3_z(d, A0.x, A0.y, A0.z, A0.w, h ? Hb[j].z : Hb[j].x, h ? Hb[j].w : Hb[j].y);
#pragma unroll
              for (int q = 0; q < 4; ++q) tot[j][q] = fmaf(d[q], si, tot[j][q]);
            }
          }
        }
      }
    }
  } else {
    const int nch = min(4, a.I_loc / 64 - p * 4);
    uint4 A0[4], Hb[4][NTL];
    uint32_t S[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (i < nch) {
        const uint8_t* ch = stage + i * 544;
        A0[i] = lds16(ch + lane * 16);
        S[i] = lds32(ch + 512 + 4 * g);
#pragma unroll
        for (int j = 0; j < NTL; ++j) Hb[i][j] = lds16(hr[j] + i * 64);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (i < nch) fp4_chunk_mma<NTL>(A0[i], S[i], Hb[i], tot);
  }
  // hi + lo / 16, routing weight and the h pre-scale; then slot columns -> token columns
  const float fs = (FMT == DSMOE_FMT_FP4 ? kFp4E4m3Scale : 1.0f) / kHScale;
  float vg[NTL], vh[NTL];
#pragma unroll
  for (int j = 0; j < NTL; ++j) {
    const int q = 4 * j + tq;
    const float f = q < ntok ? pl.wt[s][q] * fs : 0.f;
    vg[j] = (tot[j][0] + tot[j][1] * kLoInv) * f;
    vh[j] = (tot[j][2] + tot[j][3] * kLoInv) * f;
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int tok = 2 * tq + h;
    const int col = tok < a.B ? pl.col_of[s][tok] : -1;
    const int src = g * 4 + (col < 0 ? 0 : (col & 3));
#pragma unroll
    for (int j = 0; j < NTL; ++j) {
      const float x0 = __shfl_sync(0xffffffffu, vg[j], src), x1 = __shfl_sync(0xffffffffu, vh[j], src);
      if (col >= 0 && (col >> 2) == j) {
        out[h] += x0;
        out[2 + h] += x1;
      }
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
  uint8_t* xq = ring + (size_t)a.nstage * FSTAGE;  // [B][2 terms] rows of xrs bytes
  uint64_t* full = reinterpret_cast<uint64_t*>(xq + (size_t)a.B * 2 * a.xrs);
  uint64_t* empty = full + a.nstage;
  uint64_t* planbar = empty + a.nstage;  // [0] plan ready, [1] grid barrier B passed
  FPlan& pl = *reinterpret_cast<FPlan*>(planbar + 2);
  unsigned* emask = reinterpret_cast<unsigned*>(&pl + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int G = gridDim.x, cta = blockIdx.x;
  const Geo geo = make_geo(a);
  const Span rspan = cta_span(geo.NR, cta, G), sspan = cta_span(geo.NS, cta, G);
  const int my_router = rspan.e - rspan.s;
  const Span localR = {0, my_router + sspan.e - sspan.s};  // phase R: router part, then shared part

  if (tid == 0) {
    for (int s = 0; s < a.nstage; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&planbar[0], 1);
    mbar_init(&planbar[1], 1);
    pl.router_done = 0;
    pl.abort = 0;
    fence_mbar_init();
  }
  __syncthreads();

  // ================================================================ producer warp
  // Lane w (< FW) feeds consumer warp w: it walks the same runs in the same order and fills the
  // warp's own stages (w * spw .. w * spw + spw - 1), so every stage has one issuer and one reader.
  const int spw = a.nstage / FW;  // stages per consumer warp
  if (warp == FW) {
    if (lane >= FW) return;
    const int w = lane;
    int kw = 0;  // items issued for warp w
    bool ok = true;
    int def_n = 0, def_stage[2], def_slot[2], def_p[2];  // w2 items waiting for their h rows
    bool h_open = false;
    int kw2 = 0x7FFFFFFF;  // item number of warp w's first w2 item
    auto copy_h = [&](int st, int slot, int p) {  // the slot's hi rows and lo rows of part p
      const int sidx = slot < pl.n_routed ? slot : a.sh_idx;
      const uint32_t nb = (uint32_t)(pl.ntok[slot] * kHPartK);
      const uint8_t* src = a.hq + (long long)sidx * hq_slot_bytes(a.I_loc) + (long long)p * kHPartBytes;
      uint8_t* dst = ring + (size_t)st * FSTAGE + FH2;
      bulk_g2s(dst, src, nb, &full[st]);
      bulk_g2s(dst + FH2T, src + 8 * kHPartK, nb, &full[st]);
    };
    auto open_h = [&]() {  // grid barrier B passed: h is complete; send the deferred h rows
      if (h_open || !ok) return;
      if (!mbar_wait(&planbar[1], 0, 4 * kWaitNs)) {
        atomicOr(a.status, ST_PLAN);
        ok = false;
        return;
      }
      asm volatile("fence.proxy.async.global;" ::: "memory");
      for (int d = 0; d < def_n; ++d) copy_h(def_stage[d], def_slot[d], def_p[d]);
      h_open = true;
    };
    auto acquire = [&](int& st) -> bool {  // warp w's next stage, free
      st = w * spw + kw % spw;
      const int f = kw / spw;
      if (f > 0) {
        if (kw - spw >= kw2) open_h();  // its last occupant was a w2 item: it needs its h rows first
        if (!ok) return false;
        if (!mbar_wait(&empty[st], (f - 1) & 1, kWaitNs)) {
          atomicOr(a.status, ST_EMPTY);
          ok = false;
          return false;
        }
      }
      return true;
    };
    auto issue = [&](const void* src, uint32_t bytes) {
      int st;
      if (!ok || !acquire(st)) return;
      mbar_expect_tx(&full[st], bytes);
      bulk_g2s(ring + (size_t)st * FSTAGE, src, bytes, &full[st]);
      ++kw;
    };
    // phase R
    {
      const Span run = warp_run(localR, w);
      for (int li = run.s; li < run.e && ok; ++li) {
        if (li < my_router) {
          const int i = rspan.s + li;
          issue(a.wg + (long long)(i >> 2) * a.H + (i & 3) * (a.H / 4), (uint32_t)a.H);
        } else {
          const int i = sspan.s + li - my_router, t = i / geo.P13s, p = i % geo.P13s;
          issue(a.s_w13 + t * geo.tile13s + (long long)p * kFp8W13Item, kFp8W13Item);
        }
      }
    }
    if (ok && !mbar_wait(&planbar[0], 0, 4 * kWaitNs)) {
      atomicOr(a.status, ST_PLAN);
      ok = false;
    }
    if (ok) {
      const int nr = pl.n_routed;
      const int N1 = nr * geo.T * geo.P13r;
      {  // phase 1: walk the run incrementally (tile, part)
        const Span run = warp_run(cta_span(N1, cta, G), w);
        int tile = run.s / geo.P13r, p = run.s % geo.P13r;
        const uint32_t ib = RFMT == DSMOE_FMT_FP8 ? kFp8W13Item : FCH * 1088;
        for (int i = run.s; i < run.e && ok; ++i) {
          const int sl = tile / geo.T, t = tile - sl * geo.T;
          issue(a.r_w13 + (long long)pl.expert[sl] * a.r_w13_eb + t * geo.tile13r + (long long)p * ib, ib);
          if (++p == geo.P13r) {
            p = 0;
            ++tile;
          }
        }
      }
      {  // phase 2: (n-tile, slot, part), h rows deferred until grid barrier B
        const int Q = (nr + 1) * geo.P2;
        const Span run = warp_run(cta_span(geo.NT * Q, cta, G), w);
        kw2 = kw;
        int nt = run.s / Q, jq = run.s % Q;
        for (int i = run.s; i < run.e && ok; ++i) {
          const int sl = jq / geo.P2, p = jq - sl * geo.P2;
          int st;
          if (!acquire(st)) break;
          const uint32_t hbytes = (uint32_t)(2 * pl.ntok[sl] * kHPartK);
          const uint8_t* src;
          uint32_t bytes;
          if (sl < nr && RFMT == DSMOE_FMT_FP4) {
            const int nch = min(4, a.I_loc / 64 - p * 4);
            src = a.r_w2 + (long long)pl.expert[sl] * a.r_w2_eb + nt * geo.tile2r + (long long)p * 4 * 544;
            bytes = (uint32_t)(nch * 544);
          } else {
            const uint8_t* tile = sl < nr ? a.r_w2 + (long long)pl.expert[sl] * a.r_w2_eb + nt * geo.tile2r
                                          : a.s_w2 + nt * geo.tile2s;
            const int nch = min(8, a.I_loc / 32 - p * 8);
            src = tile + (long long)p * kFp8W2Item;
            bytes = (uint32_t)(nch * 512 + 32);
          }
          mbar_expect_tx(&full[st], bytes + hbytes);
          bulk_g2s(ring + (size_t)st * FSTAGE, src, bytes, &full[st]);
          if (h_open) {
            copy_h(st, sl, p);
          } else {
            def_stage[def_n] = st;
            def_slot[def_n] = sl;
            def_p[def_n] = p;
            ++def_n;
          }
          ++kw;
          if (++jq == Q) {
            jq = 0;
            ++nt;
          }
        }
      }
      open_h();
    }
    // let every copy this lane issued land before the CTA may exit
    for (int q = max(0, kw - spw); q < kw; ++q) mbar_wait(&full[w * spw + q % spw], (q / spw) & 1, kWaitNs);
    return;
  }

  // ================================================================ consumer warps
  // token rows: amax -> power-of-2 pre-scale (amax * 2^-p in [128, 256)) -> e4m3 hi / lo rows in
  // shared memory, K in B-operand order (qk_off); one pass of loads, all in flight at once
  for (int b = warp; b < a.B; b += FW) {
    const __nv_bfloat16* xr = a.x + (long long)b * a.H;
    const int nchunk = a.H / 32;  // <= 256: at most 8 chunks of 32 values per lane
    float m = 0.f;
#pragma unroll
    for (int k0 = 0; k0 < 8; k0 += 4) {  // 4 chunks (16 loads) in flight per batch
      uint4 u[4][4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int c = lane + 32 * (k0 + k);
        if (c < nchunk) {
#pragma unroll
          for (int q = 0; q < 4; ++q) u[k][q] = __ldg(reinterpret_cast<const uint4*>(xr + 32 * c + 8 * q));
        }
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (lane + 32 * (k0 + k) < nchunk) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t w[4] = {u[k][q].x, u[k][q].y, u[k][q].z, u[k][q].w};
#pragma unroll
            for (int h = 0; h < 4; ++h)
              m = fmaxf(m, fmaxf(fabsf(__uint_as_float(w[h] << 16)), fabsf(__uint_as_float(w[h] & 0xFFFF0000u))));
          }
        }
      }
    }
    m = warp_max(m);
    int p = 0;
    if (m > 0.f && m <= 3.0e38f) {
      int e2;
      frexpf(m, &e2);
      p = e2 - 8;
    }
    if (lane == 0) pl.xscale[b] = ldexpf(1.0f, p);
    const float inv = ldexpf(1.0f, -p);
    uint8_t* rh = xq + (size_t)(2 * b) * a.xrs;
    uint8_t* rl = rh + a.xrs;
#pragma unroll
    for (int k0 = 0; k0 < 8; k0 += 4) {  // second pass over the (now cached) row: convert
      uint4 u[4][4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int c = lane + 32 * (k0 + k);
        if (c < nchunk) {
#pragma unroll
          for (int q = 0; q < 4; ++q) u[k][q] = __ldg(reinterpret_cast<const uint4*>(xr + 32 * c + 8 * q));
        }
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int c = lane + 32 * (k0 + k);
        if (c < nchunk) {
          float v[32];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t w[4] = {u[k][q].x, u[k][q].y, u[k][q].z, u[k][q].w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              v[8 * q + 2 * h] = __uint_as_float(w[h] << 16) * inv;
              v[8 * q + 2 * h + 1] = __uint_as_float(w[h] & 0xFFFF0000u) * inv;
            }
          }
#pragma unroll
          for (int tt = 0; tt < 4; ++tt) {  // lane tt's 8 bytes of this 32-K chunk, per term
            uint32_t h0, l0, h1, l1, h2, l2, h3, l3;
            split2_e4m3(v[4 * tt], v[4 * tt + 1], h0, l0);
            split2_e4m3(v[4 * tt + 2], v[4 * tt + 3], h1, l1);
            split2_e4m3(v[16 + 4 * tt], v[16 + 4 * tt + 1], h2, l2);
            split2_e4m3(v[16 + 4 * tt + 2], v[16 + 4 * tt + 3], h3, l3);
            const int off = (c >> 1) * 64 + tt * 16 + (c & 1) * 8;
            *reinterpret_cast<uint2*>(rh + off) = make_uint2(h0 | (h1 << 16), h2 | (h3 << 16));
            *reinterpret_cast<uint2*>(rl + off) = make_uint2(l0 | (l1 << 16), l2 | (l3 << 16));
          }
        }
      }
    }
  }
  for (int e = tid; e < a.E; e += FW * 32) emask[e] = 0u;
  if (my_router == 0 && tid == 0) pl.gen_a = grid_arrive(a.gbar, G);
  named_bar_sync(1, FW * 32);

  int shared_toks[FMAXB];
#pragma unroll
  for (int b = 0; b < FMAXB; ++b) shared_toks[b] = min(b, a.B - 1);
  // the lane's token row (B column g) of n-tile j, for a slot's token list
  auto token_rows = [&](const uint8_t** xr, const int* toks, int ntok) {
#pragma unroll
    for (int j = 0; j < 2; ++j)
      xr[j] = xq + (size_t)(2 * toks[min(4 * j + (lane >> 3), ntok - 1)] + ((lane >> 2) & 1)) * a.xrs +
              (lane & 3) * 16;
  };

  int kw = 0;  // this warp's items so far: stage warp * spw + kw % spw, fill kw / spw
  auto stage_of = [&]() { return ring + (size_t)(warp * spw + kw % spw) * FSTAGE; };
  auto wait_full = [&]() -> bool {
    if (*(volatile int*)&pl.abort) return false;
    if (!mbar_wait(&full[warp * spw + kw % spw], (kw / spw) & 1, kWaitNs)) {
      if (lane == 0) {
        atomicOr(a.status, ST_FULL);
        pl.abort = 1;
      }
      return false;
    }
    return true;
  };
  auto release = [&]() {
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[warp * spw + kw % spw]);
    ++kw;
  };

  // ---- phase R: router quarter-rows, then the shared expert's w1|w3 parts
  {
    const Span run = warp_run(localR, warp);
    int cur = -1, seg_first = 0, seg_np = 0, n_router = 0;
    float acc1[2][4], acc3[2][4];
    const uint8_t* xr[2];
    token_rows(xr, shared_toks, a.B);
    auto flush = [&]() {
      w13_flush(a, geo, pl, geo.P13s, seg_first - cur * geo.P13s, seg_np, a.sh_idx, cur, acc1, acc3, a.B, shared_toks,
                1.0f, lane, [&](auto&& f) {
                  for_segments_R(geo.NR, geo.NS, G, cur * geo.P13s, (cur + 1) * geo.P13s, f);
                });
    };
    for (int li = run.s; li < run.e; ++li) {
      if (!wait_full()) break;
      const uint8_t* stage = stage_of();
      if (li < my_router) {
        const int i = rspan.s + li;
        router_item(a, stage, i >> 2, i & 3, lane);
        ++n_router;
      } else {
        const int i = sspan.s + li - my_router, t = i / geo.P13s, p = i % geo.P13s;
        if (t != cur) {
          if (cur >= 0) flush();
          cur = t;
          seg_first = i;
          seg_np = 0;
#pragma unroll
          for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc1[j][q] = acc3[j][q] = 0.f;
        }
        if (a.B > 4)
          w13_accum<DSMOE_FMT_FP8, 2>(stage, xr, p, lane, acc1, acc3);
        else
          w13_accum<DSMOE_FMT_FP8, 1>(stage, xr, p, lane, acc1, acc3);
        ++seg_np;
      }
      release();
      if (li + 1 == min(run.e, my_router)) {  // this warp's last router row: count its rows toward barrier A
        __threadfence();
        __syncwarp();
        if (lane == 0) {
          const unsigned done = atomicAdd(&pl.router_done, (unsigned)n_router) + n_router;
          if ((int)done == my_router) pl.gen_a = grid_arrive(a.gbar, G);
        }
      }
    }
    if (cur >= 0 && !pl.abort) flush();
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
  __threadfence();

  // ---- plan: identical in every CTA. The ring is idle here (phase R consumed, phase 1 not yet
  // issued), so its first bytes hold the scores.
  {
    float* sc_s = reinterpret_cast<float*>(ring);    // [B][E] scores
    float* bi_s = sc_s + a.B * a.E;                  // [B][E] scores + selection bias
    const int n = a.B * a.E;
    for (int i0 = tid; i0 < n; i0 += 4 * FW * 32) {
      double l4[4][4];
      float bs[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * FW * 32;
        if (i < n) {
          const int b = i / a.E, e = i % a.E;
          const double* r4 = a.rl + (long long)i * 4;
#pragma unroll
          for (int q = 0; q < 4; ++q) l4[u][q] = ld_cg_f64(r4 + q);
          const bool vl = a.bias_vl != nullptr && a.image_mask != nullptr && a.image_mask[b] != 0;
          bs[u] = (vl ? a.bias_vl : a.bias)[e];
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * FW * 32;
        if (i < n) {
          const float sc = fscore(__double2float_rn(((l4[u][0] + l4[u][1]) + l4[u][2]) + l4[u][3]), a.score_func);
          sc_s[i] = sc;
          bi_s[i] = sc + bs[u];
        }
      }
    }
    named_bar_sync(1, FW * 32);
    if (cta == 0 && a.scores)
      for (int i = tid; i < n; i += FW * 32) a.scores[i] = sc_s[i];
    for (int b = warp; b < a.B; b += FW) {  // top-k of token b: lane-local top-k lists, then k warp argmaxes
      float tv[FMAXK];
      int ti[FMAXK];
#pragma unroll
      for (int r = 0; r < FMAXK; ++r) {
        tv[r] = -INFINITY;
        ti[r] = 0x7FFFFFFF;
      }
      for (int e = lane; e < a.E; e += 32) {
        float v = bi_s[b * a.E + e];
        int vi = e;
#pragma unroll
        for (int r = 0; r < FMAXK; ++r) {  // insertion: larger value first, lower index on ties
          if (v > tv[r] || (v == tv[r] && vi < ti[r])) {
            const float ov = tv[r];
            const int oi = ti[r];
            tv[r] = v;
            ti[r] = vi;
            v = ov;
            vi = oi;
          }
        }
      }
      float tot = 0.f;
      for (int r = 0; r < a.topk; ++r) {
        float best = tv[0];
        int bi = ti[0];
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
        if (ti[0] == bi) {  // the winning lane pops its head
#pragma unroll
          for (int q = 0; q < FMAXK - 1; ++q) {
            tv[q] = tv[q + 1];
            ti[q] = ti[q + 1];
          }
          tv[FMAXK - 1] = -INFINITY;
          ti[FMAXK - 1] = 0x7FFFFFFF;
        }
        const float w = sc_s[b * a.E + bi];
        if (lane == 0) {
          pl.sel[b][r] = bi;
          pl.selw[b][r] = w;
        }
        tot += w;
      }
      __syncwarp();
      if (lane < a.topk) {
        const float w = pl.selw[b][lane] / (tot + 1e-20f) * a.route_scale;
        pl.selw[b][lane] = w;
        if (cta == 0) {
          if (a.idx) a.idx[b * a.topk + lane] = pl.sel[b][lane];
          if (a.wt) a.wt[b * a.topk + lane] = w;
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
  if (tid == 0) mbar_arrive(&planbar[0]);

  // ---- phase 1: routed w1|w3
  const int nr = pl.n_routed;
  const int N1 = nr * geo.T * geo.P13r;
  {
    const Span span = cta_span(N1, cta, G);
    const Span run = warp_run(span, warp);
    int cur = -1, seg_first = 0, seg_np = 0;
    float acc1[2][4], acc3[2][4];
    const uint8_t* xr[2];
    constexpr float fmtf = RFMT == DSMOE_FMT_FP4 ? kFp4E4m3Scale : 1.0f;
    auto flush = [&]() {
      const int cs = cur / geo.T;
      w13_flush(a, geo, pl, geo.P13r, seg_first - cur * geo.P13r, seg_np, cs, cur % geo.T, acc1, acc3, pl.ntok[cs],
                pl.tok[cs], fmtf, lane,
                [&](auto&& f) { for_segments(N1, G, cur * geo.P13r, (cur + 1) * geo.P13r, f); });
    };
    for (int i = run.s; i < run.e; ++i) {
      if (!wait_full()) break;
      const uint8_t* stage = stage_of();
      const int tile = i / geo.P13r, p = i % geo.P13r, s = tile / geo.T;
      if (tile != cur) {
        if (cur >= 0) flush();
        cur = tile;
        seg_first = i;
        seg_np = 0;
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int q = 0; q < 4; ++q) acc1[j][q] = acc3[j][q] = 0.f;
        token_rows(xr, pl.tok[s], pl.ntok[s]);
      }
      if (pl.ntok[s] > 4)
        w13_accum<RFMT, 2>(stage, xr, p, lane, acc1, acc3);
      else
        w13_accum<RFMT, 1>(stage, xr, p, lane, acc1, acc3);
      ++seg_np;
      release();
    }
    if (cur >= 0 && !pl.abort) flush();
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
  if (tid == 0 && !pl.abort) mbar_arrive(&planbar[1]);  // the producer may now copy h rows
  if (pl.abort) return;

  // ---- phase 2: w2
  {
    const int Q = (nr + 1) * geo.P2;
    const int N2 = geo.NT * Q;
    const Span span = cta_span(N2, cta, G);
    const Span run = warp_run(span, warp);
    int cur = -1, seg_first = 0, seg_np = 0;
    float out[4] = {0.f, 0.f, 0.f, 0.f};
    for (int i = run.s; i < run.e; ++i) {
      if (!wait_full()) break;
      const uint8_t* stage = stage_of();
      const int nt = i / Q, jq = i % Q, s = jq / geo.P2, p = jq % geo.P2;
      if (nt != cur) {
        if (cur >= 0) w2_flush(a, N2, Q, cur, seg_first, seg_np, out, lane);
        cur = nt;
        seg_first = i;
        seg_np = 0;
        out[0] = out[1] = out[2] = out[3] = 0.f;
      }
      const bool two = pl.ntok[s] > 4;
      if (s < nr) {
        if (two)
          w2_accum<RFMT, 2>(a, pl, stage, s, p, lane, out);
        else
          w2_accum<RFMT, 1>(a, pl, stage, s, p, lane, out);
      } else {
        if (two)
          w2_accum<DSMOE_FMT_FP8, 2>(a, pl, stage, s, p, lane, out);
        else
          w2_accum<DSMOE_FMT_FP8, 1>(a, pl, stage, s, p, lane, out);
      }
      ++seg_np;
      release();
    }
    if (cur >= 0 && !pl.abort) w2_flush(a, N2, Q, cur, seg_first, seg_np, out, lane);
  }
}

// ------------------------------------------------------------------ host side
size_t fused_smem_bytes(int H, int B, int E, int nstage) {
  const size_t xrs = (size_t)H + 64;
  return (size_t)nstage * FSTAGE + (size_t)B * 2 * xrs + (2 * (size_t)nstage + 2) * 8 + sizeof(FPlan) +
         (size_t)E * 4 + 16;
}

struct FusedScratch {
  size_t rl, p13, p2, hq, cnt13, cnt2, gbar, status, total;
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
  f.hq = o; o += al2((size_t)f.slots * hq_slot_bytes(I_loc));
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
  int nstage = 2 * FW;  // two stages per consumer warp, or one when shared memory is short
  if (fused_smem_bytes(L->hidden, B, L->n_experts, nstage) > (size_t)optin) nstage = FW;
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
  a.hq = ws + f.hq;
  a.cnt13 = (unsigned*)(ws + f.cnt13);
  a.cnt2 = (unsigned*)(ws + f.cnt2);
  a.gbar = (unsigned*)(ws + f.gbar);
  a.status = (unsigned*)(ws + f.status);
  a.sh_idx = FMAXB * L->topk;
  a.nstage = nstage;
  a.xrs = L->hidden + 64;
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
