// One persistent kernel per MoE layer for decode batches of 1..8 tokens.
//
// Replaces the per-layer sequence of the reference's decode -- device router GEMV, host top-k,
// host->device control write, SlotCat gather, w1/w3/shared matmuls, Q20 SwiGLU, w2 matmuls
// (dsv41/tt/model.py:400-442; dsv41/tt/moe.py:108-180; dsv41/kernels/slot_cat.cpp) -- with one
// launch that streams every weight byte the step needs exactly once.
//
// Shape: one CTA per SM (cooperative launch), 8 warps. Every warp walks its own list of work items
// and keeps two of them in flight: lane 0 issues a 1-D bulk copy (cp.async.bulk, the TMA engine,
// L2 evict-first) of an item's packed weights and scales into one of the warp's two 8.5 KB
// shared-memory stages, counted on that stage's mbarrier, while the warp computes on the other. A
// stage is refilled by the warp that just read it. Compute reads nothing from global memory on
// the streaming path: A fragments straight from the stage (FP8 bytes as they are, FP4 expanded to
// e4m3 with integer operations), mma.sync m16n8k32 e4m3 x e4m3 -> fp32 against e4m3 hi / lo
// activation rows held in shared memory, block scales on the fp32 partials.
// A warp accumulates consecutive items of one output tile in registers and writes one partial per
// tile it shares with other warps; every sum over partials runs in a fixed order derived from the
// deterministic distribution, so results do not depend on timing.
// Phases:
//   R  router quarter-rows (fp64 accumulation), spread round-robin over the warps, each partial
//      stored with the launch's tag; then the shared expert's weights (routing-independent) are
//      prefetched into L2 and the token rows converted to e4m3 hi / lo.
//   P  every CTA polls every tagged router partial (no grid barrier) and computes the same scores,
//      top-k and slot plan (shared memory).
//   1  w1|w3 tiles (16 rows of a slot: the routed slots, then the shared expert as the last slot),
//      whole tiles per CTA; the CTA's warps split each tile's parts, and one warp (rotating) sums
//      their partials in warp order: clamp / SiLU / up -> h as e4m3 hi / lo rows in the workspace,
//      and a per-slot count of finished tiles.
//   2  w2 items (slot, 16 output rows, 512 K of FP8 or 1024 K of FP4), slot-major, so a CTA touches
//      at most two slots: once their tiles are counted it copies their h rows into shared memory.
//      Routing weight on the fp32 partials; after grid barrier C every warp of the grid sums the
//      slots' partials of (at most a few) 16-row output tiles into y.
// Every wait (mbarrier, grid barrier, slot count) is bounded by %globaltimer; on expiry the kernel
// records a status bit in the workspace, stops consuming, lets its own copies land and returns.
#include "exchange.cuh"

namespace dsmoe {

constexpr int FW = 8;                  // warps per CTA
constexpr int FT = FW * 32;
constexpr int SPW = 2;                 // stages per warp
constexpr int NST = FW * SPW;
constexpr int FCH = 8;                 // packed chunks per w1|w3 item
constexpr int FSTAGE = FCH * 1088;     // bytes per stage (8 FP4 w1|w3 chunks, the largest item)
constexpr int FK2_8 = 512;             // K per FP8 w2 item: two 8-chunk store items (8256 B)
constexpr int FK2_4 = 1024;            // K per FP4 w2 item: 16 chunks of 544 B (8704 B)
static_assert(2 * kFp8W2Item <= FSTAGE && 16 * 544 <= FSTAGE, "w2 item exceeds a stage");
constexpr int FMAXB = 8;               // tokens per call
constexpr int FXB = 4;                 // up to this many tokens keep bf16 x in shared memory (router)
constexpr int FMAXK = DSMOE_MAX_TOPK;
constexpr int FMAXS = FMAXB * FMAXK + 1;
constexpr int FEMAX = 1024;            // routed experts
constexpr int FHSLOTS = 2;             // slots whose h rows a CTA stages for phase 2
constexpr int NPEND = 8;               // segments a warp holds before publishing them (published-segment phase 1)
constexpr int kMaxCtas = 256;          // CTAs (one per SM) the phase-1 partial scratch is sized for
constexpr uint64_t kWaitNs = 1000000000ull;
constexpr uint64_t kPeerWaitNs = 5000000000ull;  // a peer GPU's tile: ranks may start seconds apart

enum : unsigned { ST_FULL = 1u, ST_SLOT = 2u, ST_GRID = 8u, ST_PEER = 16u };

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
  unsigned long long* rl;  // [8][E][4] router quarter-row partial logits, two epoch-tagged words each
  float* p13;          // [CTA][2 parities][FW warps][32][8] w1|w3 partials of the CTA's current tiles
  float* p2;           // [NT][slots][p2max][32][4] w2 segment partials (token columns)
  uint8_t* hq;         // [slots] h rows, e4m3 hi / lo (hq_row)
  unsigned* cnt13;     // [slots][T]
  unsigned* cnt2;      // [NT]
  unsigned* slot_done; // [slots] finished w1|w3 tiles per routed slot
  unsigned long long* gbar;  // grid-barrier arrivals since the workspace was reset
  unsigned* status;    // [0]
  int sh_idx;          // scratch slot index of the shared expert
  int slots, p13max, p2max;
  // peer all-reduce of y (ar_world > 1): see ar_tile
  int ar_world, ar_rank;
  unsigned* ar_ctl;
  unsigned long long* ar_slots[kMaxWorld];
};

struct FPlan {
  int n_routed;
  int expert[FMAXS];
  int ntok[FMAXS];
  int tok[FMAXS][8];
  float wt[FMAXS][8];
  signed char col_of[FMAXS][8];
  float xscale[FMAXB];
  float xinv[FMAXB];
  float red[FW][FMAXB];
  int sel[FMAXB][FMAXK];
  float selw[FMAXB][FMAXK];
  int wcnt[FW];
  int abort;
  unsigned ar_epoch;
  unsigned rl_epoch;  // this launch's tag on the router partials
};

// Shared-memory carve-up (host and device agree): stage ring; token rows (e4m3 hi rows [B][H], lo
// rows [B][H] 64 bytes further) and bf16 token rows for the router (B <= FXB), a region that phase 2
// reuses for the h rows of up to FHSLOTS slots; stage mbarriers + the h mbarrier; plan; per-expert
// token masks.
struct SmemLayout {
  size_t xq, xs, hs_stride, bars, plan, emask, total;
};
__host__ __device__ inline SmemLayout smem_layout(int H, int I_loc, int B, int E) {
  SmemLayout L;
  size_t o = (size_t)NST * FSTAGE;
  L.xq = o;
  const size_t xbytes = 2 * (size_t)B * H + 64 + (B <= FXB ? (size_t)B * H * 2 : 0);
  L.xs = o + 2 * (size_t)B * H + 64;
  L.hs_stride = 2 * (size_t)B * hq_row_bytes(I_loc) + 64;
  const size_t hbytes = FHSLOTS * L.hs_stride;
  o += xbytes > hbytes ? xbytes : hbytes;
  o = (o + 15) & ~size_t(15);
  L.bars = o;
  o += (size_t)(NST + 6) * 8;  // stage barriers, the h barrier, the token-row barrier, 2 + 2 tile barriers
  L.plan = o;
  o += (sizeof(FPlan) + 15) & ~size_t(15);
  L.emask = o;
  o += (size_t)E * 4;
  L.total = o;
  return L;
}

struct Geo {
  int T, NT, NR, NS, P13s, P13r, P2r, P2s;
  long long tile13r, tile13s, tile2r, tile2s;
};

__device__ __forceinline__ Geo make_geo(const FusedArgs& a) {
  Geo g;
  g.T = a.I_loc / 16;
  g.NT = a.H / 16;
  g.NR = 4 * a.E;
  g.P13s = (a.H / 32) / FCH;
  g.P13r = a.r_fmt == DSMOE_FMT_FP8 ? (a.H / 32) / FCH : (a.H / 64) / FCH;
  g.NS = g.T * g.P13s;
  g.P2r = a.r_fmt == DSMOE_FMT_FP8 ? (a.I_loc + FK2_8 - 1) / FK2_8 : (a.I_loc + FK2_4 - 1) / FK2_4;
  g.P2s = (a.I_loc + FK2_8 - 1) / FK2_8;
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
// n * G stays below 2^31 for every item space of a supported layer (checked on the host), so the
// split uses 32-bit unsigned division.
__host__ __device__ __forceinline__ Span cta_span(int n, int c, int G) {
  return {(int)((unsigned)n * (unsigned)c / (unsigned)G), (int)((unsigned)n * (unsigned)(c + 1) / (unsigned)G)};
}
__device__ __forceinline__ Span warp_run(Span cs, int w) {
  const int nc = cs.e - cs.s, L = nc / FW, r = nc % FW;
  const int rs = cs.s + w * L + min(w, r);
  return {rs, rs + L + (w < r ? 1 : 0)};
}
// Split of an item space whose first n1 items (routed experts) cost w1 each and the other n - n1
// (the shared expert) w2: CTA c takes the items whose cost position falls in [c C / G, (c+1) C / G),
// C the total cost. With FP4 routed experts an item holds twice the weights of a shared FP8 item,
// so w1 = 2, w2 = 1 gives every CTA the same work; 2 n G < 2^32 (host check) keeps it 32-bit.
struct Split {
  int n, n1, w1, w2;
  __device__ __forceinline__ int bound(int c, int G) const {
    const unsigned C = (unsigned)n1 * w1 + (unsigned)(n - n1) * w2;
    const unsigned q = (unsigned)c * C, a1 = (unsigned)n1 * w1 * (unsigned)G;
    const unsigned g1 = (unsigned)w1 * G, g2 = (unsigned)w2 * G;
    if (q <= a1) return (int)((q + g1 - 1) / g1);
    return min(n, n1 + (int)((q - a1 + g2 - 1) / g2));
  }
  __device__ __forceinline__ Span span(int c, int G) const { return {bound(c, G), bound(c + 1, G)}; }
  __device__ __forceinline__ int first_cta(int i, int G) const {  // a guess, refined by the caller
    const unsigned C = (unsigned)n1 * w1 + (unsigned)(n - n1) * w2;
    const unsigned pos = i < n1 ? (unsigned)i * w1 : (unsigned)n1 * w1 + (unsigned)(i - n1) * w2;
    return C ? (int)(((unsigned long long)pos * G) / C) : 0;
  }
};
// Item i of the split belongs to CTA span / warp run as above. Calls f(first item of the segment -
// a) for every warp run that intersects [a, b), in order.
template <class F>
__device__ __forceinline__ void for_segments(const Split& sp, int G, int a, int b, F&& f) {
  int c = min(sp.first_cta(a, G), G - 1);
  while (c + 1 < G && sp.span(c + 1, G).s <= a) ++c;
  while (c > 0 && sp.span(c, G).s > a) --c;
  for (; c < G; ++c) {
    const Span cs = sp.span(c, G);
    if (cs.s >= b) break;
    for (int w = 0; w < FW; ++w) {
      const Span r = warp_run(cs, w);
      if (r.e <= a || r.s >= r.e) continue;
      if (r.s >= b) break;
      f(max(r.s, a) - a);
    }
  }
}

// Phase-2 item space: routed slots first (NT x P2r items each), then the shared slot (NT x P2s),
// (slot, 16-row n-tile, part) with the part fastest.
struct W2Item {
  int s, nt, p;
};
__device__ __forceinline__ W2Item w2_item(const Geo& g, int nr, int i) {
  W2Item w;
  const int NR2 = nr * g.NT * g.P2r;
  if (i < NR2) {
    w.s = i / (g.NT * g.P2r);
    const int r = i - w.s * g.NT * g.P2r;
    w.nt = r / g.P2r;
    w.p = r - w.nt * g.P2r;
  } else {
    w.s = nr;
    const int r = i - NR2;
    w.nt = r / g.P2s;
    w.p = r - w.nt * g.P2s;
  }
  return w;
}
__device__ __forceinline__ int w2_range_start(const Geo& g, int nr, int s, int nt) {
  return s < nr ? (s * g.NT + nt) * g.P2r : nr * g.NT * g.P2r + nt * g.P2s;
}

// Position of a warp's item in the phase-2 item space, advanced without divisions:
// (slot s, n-tile t, part p). Routed slots come
// first; slot nr is the shared expert, with its own part count.
struct Cursor {
  int s, t, p;
  __device__ __forceinline__ void next(int nr, int n_t, int pr, int ps) {
    if (++p == (s < nr ? pr : ps)) {
      p = 0;
      if (++t == n_t) {
        t = 0;
        ++s;
      }
    }
  }
};
__device__ __forceinline__ Cursor cursor1(const Geo& g, int nr, int NR1, int i) {
  Cursor c;
  if (i < NR1) {
    const int tile = i / g.P13r;
    c.p = i - tile * g.P13r;
    c.s = tile / g.T;
    c.t = tile - c.s * g.T;
  } else {
    const int j = i - NR1;
    c.t = j / g.P13s;
    c.p = j - c.t * g.P13s;
    c.s = nr;
  }
  return c;
}
__device__ __forceinline__ Cursor cursor2(const Geo& g, int nr, int i) {
  const W2Item w = w2_item(g, nr, i);
  return {w.s, w.nt, w.p};
}

// Phase 1: each CTA owns whole w1|w3 tiles, tile tau over [routed slots' tiles (slot-major), the
// shared slot's tiles]; its span is cta_span(tiles, cta, G). The warps split every owned tile's P
// parts into FW runs [P j / FW, P (j + 1) / FW); warp w takes run j = (w + k) % FW of tile k, so the
// longer runs rotate over the warps. TCursor walks a warp's parts, tile k of the span.
__device__ __forceinline__ int tile_nparts(const Geo& g, int nr, int tau) { return tau < nr * g.T ? g.P13r : g.P13s; }
__device__ __forceinline__ int run_of(int w, int k) { return (w + k) % FW; }
struct TCursor {
  int k, p;
  // to the warp's next part, skipping tiles where it has none (k == ntl at the end)
  __device__ __forceinline__ void next(const Geo& g, int nr, int tau0, int ntl, int w) {
    ++p;
    while (k < ntl) {
      const int P = tile_nparts(g, nr, tau0 + k);
      if (p < P * (run_of(w, k) + 1) / FW) return;
      if (++k < ntl) p = tile_nparts(g, nr, tau0 + k) * run_of(w, k) / FW;
    }
  }
  __device__ __forceinline__ void start(const Geo& g, int nr, int tau0, int ntl, int w) {
    k = 0;
    p = (ntl > 0 ? tile_nparts(g, nr, tau0) * run_of(w, 0) / FW : 0) - 1;
    next(g, nr, tau0, ntl, w);
  }
};

__device__ __forceinline__ float fscore(float l, int func) {
  const double d = (double)l;
  const double s = func == DSMOE_SCORE_SIGMOID ? 1.0 / (1.0 + exp(-d)) : sqrt(d > 20.0 ? d : log1p(exp(d)));
  return __double2float_rn(s);
}

__device__ __forceinline__ uint4 lds16(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ float ldsf(const uint8_t* p) { return *reinterpret_cast<const float*>(p); }

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }

__device__ __forceinline__ uint32_t ld_relaxed_u32(const unsigned* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// ------------------------------------------------------------------ grid barrier (bounded)
// One 64-bit arrival counter per workspace, zeroed when the workspace is reset and otherwise only
// increased: each barrier of each launch adds G (one arrival per CTA). Barrier j of a launch is
// complete once the counter reaches base + (j + 1) G, where base is the counter read at launch start
// rounded down to a multiple of G: every earlier launch added a multiple of G, and fewer than G
// arrivals of this launch can precede any CTA's read (its own is missing). base / G therefore
// numbers the launches on a workspace, which tags the router partials (see rl_store).
// Arrive: a gpu-scope fence (the CTA's writes, ordered by the caller's __syncthreads) and a relaxed
// add, so the arriving thread waits for no reply. Wait: relaxed polling, one acquire fence at the end.
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long grid_base(const unsigned long long* gbar, int G) {
  const unsigned long long c = ld_relaxed_u64(gbar);
  return c - c % (unsigned long long)G;
}
__device__ __forceinline__ void grid_arrive(unsigned long long* gbar) {
  fence_acq_rel_gpu();
  asm volatile("red.relaxed.gpu.global.add.u64 [%0], 1;" ::"l"(gbar) : "memory");
}
__device__ __forceinline__ bool grid_wait(const unsigned long long* gbar, unsigned long long target,
                                          const unsigned* status) {
  const uint64_t t0 = globaltimer_ns();
  while ((long long)(ld_relaxed_u64(gbar) - target) < 0) {
    if (ld_relaxed_u32(status) != 0u) return false;
    if (globaltimer_ns() - t0 > kWaitNs) return false;
  }
  fence_acq_rel_gpu();
  return true;
}

// ------------------------------------------------------------------ top-k
// Order-preserving key of a score (a larger score has a larger key, -0 and +0 the same one); NaN
// gets the lowest key, 0, like an expert that does not exist, so it is never preferred.
__device__ __forceinline__ unsigned score_key(float f) {
  const unsigned u = f == 0.f ? 0u : __float_as_uint(f);
  return f != f ? 0u : u ^ ((unsigned)((int)u >> 31) | 0x80000000u);
}
constexpr int FKJ = 12;  // keys per lane covering 384 experts

// Top-k of one token by one warp: keys of v[e] (scores + selection bias) for e = lane + 32 j, k
// rounds of lane-local best (a tree over the lane's keys, the lower j winning a tie), warp max,
// then the lowest index holding it (ties -> lower index); the winner's lane drops it. Lane r keeps
// round r's pick; sel[r] / selw[r] (= sc[pick]) are written by lane r after the rounds, and tot is
// the sum of the k selected scores in round order.
template <int NJ>
__device__ __forceinline__ void topk_token(const float* v, const float* sc, int E, int k, int lane, int* sel,
                                           float* selw, float& tot) {
  unsigned key[NJ];
#pragma unroll
  for (int j = 0; j < NJ; ++j) key[j] = lane + 32 * j < E ? score_key(v[lane + 32 * j]) : 0u;
  unsigned mine = 0u;
  for (int r = 0; r < k; ++r) {
    unsigned bk[NJ];
    int bj[NJ];
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      bk[j] = key[j];
      bj[j] = j;
    }
#pragma unroll
    for (int w = 1; w < NJ; w *= 2)
#pragma unroll
      for (int j = 0; j + w < NJ; j += 2 * w)
        if (bk[j + w] > bk[j]) {  // strict: the lower j keeps a tie
          bk[j] = bk[j + w];
          bj[j] = bj[j + w];
        }
    const unsigned m = __reduce_max_sync(0xffffffffu, bk[0]);
    unsigned bi = __reduce_min_sync(0xffffffffu, bk[0] == m ? (unsigned)(lane + 32 * bj[0]) : 0xFFFFFFFFu);
    if (bi >= (unsigned)E) bi = 0u;  // no expert left (k > E, rejected by the host)
    if (lane == r) mine = bi;
    if (lane == (int)(bi & 31u)) {
#pragma unroll
      for (int j = 0; j < NJ; ++j)
        if (j == (int)(bi >> 5)) key[j] = 0u;
    }
  }
  const float w = lane < k ? sc[mine] : 0.f;
  if (lane < k) {
    sel[lane] = (int)mine;
    selw[lane] = w;
  }
  tot = 0.f;
  for (int r = 0; r < k; ++r) tot += __shfl_sync(0xffffffffu, w, r);
}

// ------------------------------------------------------------------ router partials
// A router partial (fp64) is two 8-byte words, each carrying 32 bits of the value and the launch's
// tag in its high half. An aligned 8-byte store is single-copy atomic, so a reader that finds the
// tag in both words has the whole value; this replaces a grid barrier between the router and the
// plan. Tags are launch numbers + 1: a zeroed workspace never matches, and a reset zeroes the words
// with the barrier counter.
__device__ __forceinline__ void rl_store(unsigned long long* p, double v, unsigned ep) {
  const unsigned long long b = (unsigned long long)__double_as_longlong(v), t = (unsigned long long)ep << 32;
  st_ll2(p, t | (b >> 32), t | (b & 0xFFFFFFFFull));
}

// ------------------------------------------------------------------ router
// Router quarter-row: 1/4 of gate_w[r] (H/4 fp32, in the stage) . x[b] for every token, each
// product exact in fp64 and accumulated there (rounded to fp32 once, after the four quarters).
// x comes from shared memory (B <= FXB) or global memory; both through one generic pointer.
__device__ void router_item(const FusedArgs& a, const uint8_t* stage, const __nv_bfloat16* xsrc, int r, int q,
                            int lane, unsigned ep) {
  const float4* wv = reinterpret_cast<const float4*>(stage);
  const int n4 = a.H / 16;  // float4 per quarter
  for (int b0 = 0; b0 < a.B; b0 += 2) {  // two tokens at a time (one for an odd last), four chains each
    const __nv_bfloat16* x0 = xsrc + (long long)b0 * a.H + q * (a.H / 4);
    if (b0 + 1 < a.B) {
      const __nv_bfloat16* x1 = x0 + a.H;
      double acc[2][4] = {{0.0, 0.0, 0.0, 0.0}, {0.0, 0.0, 0.0, 0.0}};
#pragma unroll 2
      for (int f = lane; f < n4; f += 32) {
        const float4 w = wv[f];
        const double w0 = w.x, w1 = w.y, w2 = w.z, w3 = w.w;
        const uint2 u0 = *reinterpret_cast<const uint2*>(x0 + 4 * f);
        const uint2 u1 = *reinterpret_cast<const uint2*>(x1 + 4 * f);
        acc[0][0] = fma((double)__uint_as_float(u0.x << 16), w0, acc[0][0]);
        acc[0][1] = fma((double)__uint_as_float(u0.x & 0xFFFF0000u), w1, acc[0][1]);
        acc[0][2] = fma((double)__uint_as_float(u0.y << 16), w2, acc[0][2]);
        acc[0][3] = fma((double)__uint_as_float(u0.y & 0xFFFF0000u), w3, acc[0][3]);
        acc[1][0] = fma((double)__uint_as_float(u1.x << 16), w0, acc[1][0]);
        acc[1][1] = fma((double)__uint_as_float(u1.x & 0xFFFF0000u), w1, acc[1][1]);
        acc[1][2] = fma((double)__uint_as_float(u1.y << 16), w2, acc[1][2]);
        acc[1][3] = fma((double)__uint_as_float(u1.y & 0xFFFF0000u), w3, acc[1][3]);
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const double v = warp_sum_d((acc[j][0] + acc[j][1]) + (acc[j][2] + acc[j][3]));
        if (lane == 0) rl_store(a.rl + 2 * (((long long)(b0 + j) * a.E + r) * 4 + q), v, ep);
      }
    } else {
      double acc[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll 2
      for (int f = lane; f < n4; f += 32) {
        const float4 w = wv[f];
        const uint2 u0 = *reinterpret_cast<const uint2*>(x0 + 4 * f);
        acc[0] = fma((double)__uint_as_float(u0.x << 16), (double)w.x, acc[0]);
        acc[1] = fma((double)__uint_as_float(u0.x & 0xFFFF0000u), (double)w.y, acc[1]);
        acc[2] = fma((double)__uint_as_float(u0.y << 16), (double)w.z, acc[2]);
        acc[3] = fma((double)__uint_as_float(u0.y & 0xFFFF0000u), (double)w.w, acc[3]);
      }
      const double v = warp_sum_d((acc[0] + acc[1]) + (acc[2] + acc[3]));
      if (lane == 0) rl_store(a.rl + 2 * (((long long)b0 * a.E + r) * 4 + q), v, ep);
    }
  }
}

// ------------------------------------------------------------------ token rows
// Token rows (bf16 in shared memory for B <= FXB, else global) -> per-token power-of-2 pre-scale
// (amax * 2^-p in [128, 256)) -> e4m3 hi / lo rows in B-operand order (qk_off). All threads; ends
// with __syncthreads.
__device__ void setup_tokens(const FusedArgs& a, uint8_t* xq, __nv_bfloat16* xs, FPlan& pl, int lo_off) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nv = a.H / 8;  // uint4 per row
  for (int b = 0; b < a.B; ++b) {
    const uint4* src = reinterpret_cast<const uint4*>((a.B <= FXB ? xs : a.x) + (long long)b * a.H);
    float m = 0.f;
    for (int v = tid; v < nv; v += FT) {
      const uint4 u = src[v];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int h = 0; h < 4; ++h)
        m = fmaxf(m, fmaxf(fabsf(__uint_as_float(w[h] << 16)), fabsf(__uint_as_float(w[h] & 0xFFFF0000u))));
    }
    m = warp_max(m);
    if (lane == 0) pl.red[warp][b] = m;
  }
  __syncthreads();
  if (tid < a.B) {
    float m = 0.f;
    for (int w = 0; w < FW; ++w) m = fmaxf(m, pl.red[w][tid]);
    int p = 0;
    if (m > 0.f && m <= 3.0e38f) {
      int e2;
      frexpf(m, &e2);
      p = e2 - 8;
    }
    pl.xscale[tid] = ldexpf(1.0f, p);
    pl.xinv[tid] = ldexpf(1.0f, -p);
  }
  __syncthreads();
  const int nch = a.H / 32;
  for (int i = tid; i < a.B * nch; i += FT) {
    const int b = i / nch, c = i - b * nch;
    const uint4* src = reinterpret_cast<const uint4*>((a.B <= FXB ? xs : a.x) + (long long)b * a.H + 32 * c);
    const float inv = pl.xinv[b];
    float v[32];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 u = src[q];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        v[8 * q + 2 * h] = __uint_as_float(w[h] << 16) * inv;
        v[8 * q + 2 * h + 1] = __uint_as_float(w[h] & 0xFFFF0000u) * inv;
      }
    }
    uint8_t* rh = xq + (long long)b * a.H + (c >> 1) * 64 + (c & 1) * 8;
#pragma unroll
    for (int tt = 0; tt < 4; ++tt) {  // lane-group tt's 8 bytes of this 32-K chunk, per term
      uint32_t h0, l0, h1, l1, h2, l2, h3, l3;
      split2_e4m3(v[4 * tt], v[4 * tt + 1], h0, l0);
      split2_e4m3(v[4 * tt + 2], v[4 * tt + 3], h1, l1);
      split2_e4m3(v[16 + 4 * tt], v[16 + 4 * tt + 1], h2, l2);
      split2_e4m3(v[16 + 4 * tt + 2], v[16 + 4 * tt + 3], h3, l3);
      *reinterpret_cast<uint2*>(rh + tt * 16) = make_uint2(h0 | (h1 << 16), h2 | (h3 << 16));
      *reinterpret_cast<uint2*>(rh + lo_off + tt * 16) = make_uint2(l0 | (l1 << 16), l2 | (l3 << 16));
    }
  }
  __syncthreads();
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
    for (int blk = 0; blk < 2; ++blk) {  // two 128-K blocks, four chunks each
      uint4 X[NTL][2];
#pragma unroll
      for (int j = 0; j < NTL; ++j) {
        X[j][0] = lds16(xr[j] + (4 * p + 2 * blk) * 64);
        X[j][1] = lds16(xr[j] + (4 * p + 2 * blk + 1) * 64);
      }
      float u1[4][NTL][4], u3[4][NTL][4];  // every MMA of the block independent
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 A1 = lds16(stage + (4 * blk + c) * 1024 + lane * 16);
        const uint4 A3 = lds16(stage + (4 * blk + c) * 1024 + 512 + lane * 16);
#pragma unroll
        for (int j = 0; j < NTL; ++j) {
          const uint4 xb = X[j][c >> 1];
          const uint32_t b0 = (c & 1) ? xb.z : xb.x, b1 = (c & 1) ? xb.w : xb.y;
          mma_e4m3_z(u1[c][j], A1.x, A1.y, A1.z, A1.w, b0, b1);
          mma_e4m3_z(u3[c][j], A3.x, A3.y, A3.z, A3.w, b0, b1);
        }
      }
      const float s1 = ldsf(stage + FCH * 1024 + 4 * fp8_w13_scale_index(blk, 0));
      const float s3 = ldsf(stage + FCH * 1024 + 4 * fp8_w13_scale_index(blk, 1));
#pragma unroll
      for (int j = 0; j < NTL; ++j)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          acc1[j][q] = fmaf((u1[0][j][q] + u1[1][j][q]) + (u1[2][j][q] + u1[3][j][q]), s1, acc1[j][q]);
          acc3[j][q] = fmaf((u3[0][j][q] + u3[1][j][q]) + (u3[2][j][q] + u3[3][j][q]), s3, acc3[j][q]);
        }
    }
  } else {
#pragma unroll 1
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

// hi + lo / 16 per row: the 8 per-lane values of a w1|w3 tile segment.
__device__ __forceinline__ void w13_combine(const float (&acc1)[2][4], const float (&acc3)[2][4], float (&s)[8]) {
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    s[4 * j] = acc1[j][0] + acc1[j][1] * kLoInv;
    s[4 * j + 1] = acc1[j][2] + acc1[j][3] * kLoInv;
    s[4 * j + 2] = acc3[j][0] + acc3[j][1] * kLoInv;
    s[4 * j + 3] = acc3[j][2] + acc3[j][3] * kLoInv;
  }
}



// Ordered sum of published partials (nv floats per lane, nv = 4 or 8): the offsets (in floats, from
// base) come in distribution order; up to 8 loads are in flight at a time, added in that order.
template <int NV>
struct SegSum {
  const float* base;
  float s[NV];
  int off[8];
  int n = 0;
  __device__ explicit SegSum(const float* b) : base(b) {
#pragma unroll
    for (int j = 0; j < NV; ++j) s[j] = 0.f;
  }
  __device__ void flush() {
    uint4 v[8][NV / 4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < n)
#pragma unroll
        for (int h = 0; h < NV / 4; ++h) v[i][h] = ld_cg16(base + off[i] + 4 * h);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < n)
#pragma unroll
        for (int h = 0; h < NV / 4; ++h) {
          s[4 * h] += __uint_as_float(v[i][h].x);
          s[4 * h + 1] += __uint_as_float(v[i][h].y);
          s[4 * h + 2] += __uint_as_float(v[i][h].z);
          s[4 * h + 3] += __uint_as_float(v[i][h].w);
        }
    n = 0;
  }
  __device__ void add(int o) {
    off[n++] = o;
    if (n == 8) flush();
  }
};

__device__ __forceinline__ float* p13_slot(const FusedArgs& a, const Geo& G, int sidx, int t, int rel, int lane) {
  return a.p13 + ((((long long)sidx * G.T + t) * a.p13max + rel) * 32 + lane) * 8;
}

// Sum of a w1|w3 tile's published segments, in distribution order: the tile's items are
// [a0, a0 + P) of the phase-1 item space (N1 items).
__device__ __noinline__ void w13_reduce(const FusedArgs& a, const Geo& G, int sidx, int t, int a0, int P,
                                        const Split& sp1, int lane, float* s) {
  const float* base = p13_slot(a, G, sidx, t, 0, lane);
  SegSum<8> sum(base);
  for_segments(sp1, gridDim.x, a0, a0 + P, [&](int q) { sum.add(q * 32 * 8); });
  sum.flush();
#pragma unroll
  for (int j = 0; j < 8; ++j) s[j] = sum.s[j];
}


// ------------------------------------------------------------------ w2
// One w2 item of a slot (packed weights and scales in the stage; the slot's h rows in shared memory
// at hbase: hi rows of its ntok tokens, lo rows ntok * rp + 64 bytes further) added to tot[] in
// slot columns (per n-tile j: rows g, g+8 x hi / lo terms of slot token 4j + tq).
// FP8: the item is up to two 8-chunk store items, each followed by its 32 B of chunk scales.
template <int FMT, int NTL>
__device__ __forceinline__ void w2_accum(const FusedArgs& a, const uint8_t* stage, const uint8_t* hbase, int rp,
                                         int ntok, int p, int lane, float (&tot)[2][4]) {
  const int g = lane >> 2, tq = lane & 3;
  const uint8_t* hr[NTL];
#pragma unroll
  for (int j = 0; j < NTL; ++j)
    hr[j] = hbase + (g & 1) * (ntok * rp + 64) + min(4 * j + (g >> 1), ntok - 1) * rp + tq * 16;
  if (FMT == DSMOE_FMT_FP8) {
    const int KC = a.I_loc / 32;
#pragma unroll 1
    for (int u = 0; u < 2; ++u) {
      const int c0 = 16 * p + 8 * u;  // first chunk of this store item
      const int nch = min(8, KC - c0);
      if (nch <= 0) break;
      const uint8_t* sub = stage + u * kFp8W2Item;
      const uint8_t* sc = sub + nch * 512;
      if (nch == 8) {  // full store item: every MMA independent, then the per-chunk scales
        float d[8][NTL][4];
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          uint4 Hb[NTL];
#pragma unroll
          for (int j = 0; j < NTL; ++j) Hb[j] = lds16(hr[j] + ((c0 >> 1) + b) * 64);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint4 A0 = lds16(sub + (2 * b + h) * 512 + lane * 16);
#pragma unroll
            for (int j = 0; j < NTL; ++j)
              mma_e4m3_z(d[2 * b + h][j], A0.x, A0.y, A0.z, A0.w, h ? Hb[j].z : Hb[j].x, h ? Hb[j].w : Hb[j].y);
          }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float si = ldsf(sc + 4 * i);
#pragma unroll
          for (int j = 0; j < NTL; ++j)
#pragma unroll
            for (int q = 0; q < 4; ++q) tot[j][q] = fmaf(d[i][j][q], si, tot[j][q]);
        }
      } else {
#pragma unroll 1
        for (int i = 0; i < nch; ++i) {  // short last store item
          const int kc = c0 + i;
          const uint4 A0 = lds16(sub + i * 512 + lane * 16);
          const float si = ldsf(sc + 4 * i);
#pragma unroll
          for (int j = 0; j < NTL; ++j) {
            const uint2 hb = *reinterpret_cast<const uint2*>(hr[j] + (kc >> 1) * 64 + (kc & 1) * 8);
            float d[4];
            mma_e4m3_z(d, A0.x, A0.y, A0.z, A0.w, hb.x, hb.y);
#pragma unroll
            for (int q = 0; q < 4; ++q) tot[j][q] = fmaf(d[q], si, tot[j][q]);
          }
        }
      }
    }
  } else {
    const int c0 = 16 * p, nch = min(16, a.I_loc / 64 - c0);
#pragma unroll 1
    for (int i0 = 0; i0 < nch; i0 += 4) {
#pragma unroll
      for (int i = i0; i < i0 + 4; ++i) {
        if (i < nch) {
          const uint8_t* ch = stage + i * 544;
          const uint4 A0 = lds16(ch + lane * 16);
          const uint32_t S = lds32(ch + 512 + 4 * g);
          uint4 Hb[NTL];
#pragma unroll
          for (int j = 0; j < NTL; ++j) Hb[j] = lds16(hr[j] + (c0 + i) * 64);
          fp4_chunk_mma<NTL>(A0, S, Hb, tot);
        }
      }
    }
  }
}

// A slot's accumulated w2 partial -> token columns: hi + lo / 16, routing weight, 1 / kHScale and the
// weight-format factor; out[h] / out[2 + h] = rows g / g + 8 of token 2tq + h. Clears tot.
__device__ __forceinline__ void w2_fold(const FusedArgs& a, const FPlan& pl, int s, float fs, float (&tot)[2][4],
                                        int lane, float (&out)[4]) {
  const int g = lane >> 2, tq = lane & 3;
  const int ntok = pl.ntok[s];
  float vg[2], vh[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int q = 4 * j + tq;
    const float f = q < ntok ? pl.wt[s][q] * fs : 0.f;
    vg[j] = (tot[j][0] + tot[j][1] * kLoInv) * f;
    vh[j] = (tot[j][2] + tot[j][3] * kLoInv) * f;
#pragma unroll
    for (int k = 0; k < 4; ++k) tot[j][k] = 0.f;
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int tok = 2 * tq + h;
    const int col = tok < a.B ? pl.col_of[s][tok] : -1;
    const int src = g * 4 + (col < 0 ? 0 : (col & 3));
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float x0 = __shfl_sync(0xffffffffu, vg[j], src), x1 = __shfl_sync(0xffffffffu, vh[j], src);
      if (col >= 0 && (col >> 2) == j) {
        out[h] += x0;
        out[2 + h] += x1;
      }
    }
  }
}

__device__ __forceinline__ float* p2_slot(const FusedArgs& a, int nt, int s, int rel, int lane) {
  return a.p2 + ((((long long)nt * a.slots + s) * a.p2max + rel) * 32 + lane) * 4;
}

// Ordered sum of positions [q0, q1) of n-tile nt's w2 partials. Positions run slot-major over the
// n-tile's items (nr routed slots of P2r parts, then the shared slot's P2s); every position holds a
// partial (first item of a segment) or zero (any other item), so no segment bookkeeping is needed.
__device__ __noinline__ float4 w2_chunk_sum(const FusedArgs& a, const Geo& G, int nr, int nt, int q0, int q1,
                                            int lane) {
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  const int NRP = nr * G.P2r;
  for (int qb = q0; qb < q1; qb += 8) {
    uint4 v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int q = qb + i;
      if (q < q1) {
        const int s = q < NRP ? q / G.P2r : nr, rel = q < NRP ? q - s * G.P2r : q - NRP;
        v[i] = ld_cg16(p2_slot(a, nt, s, rel, lane));
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (qb + i < q1) {
        acc.x += __uint_as_float(v[i].x);
        acc.y += __uint_as_float(v[i].y);
        acc.z += __uint_as_float(v[i].z);
        acc.w += __uint_as_float(v[i].w);
      }
    }
  }
  return acc;
}

__device__ __forceinline__ void w2_store_y(const FusedArgs& a, int nt, float4 s4, int lane) {
  const int g = lane >> 2, tq = lane & 3;
  const float v[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
  for (int q4 = 0; q4 < 4; ++q4) {
    const int row = nt * 16 + (q4 >= 2 ? g + 8 : g), tok = 2 * tq + (q4 & 1);
    if (tok < a.B) {
      const long long o = (long long)tok * a.H + row;
      if (a.y_f32)
        reinterpret_cast<float*>(a.y)[o] = v[q4];
      else
        reinterpret_cast<__nv_bfloat16*>(a.y)[o] = __float2bfloat16_rn(v[q4]);
    }
  }
}

// A call that gave up (an expired bounded wait, in this launch or one before it on the same
// workspace: the status word stays set until dsmoe_moe_check resets it) writes NaN into the rows
// of y this CTA owns (16-row tiles nt = cta + G j), so no caller reads stale memory as a result.
__device__ __noinline__ void poison_y(const FusedArgs& a) {
  const int NT = a.H / 16, G = gridDim.x;
  for (int nt = blockIdx.x; nt < NT; nt += G)
    for (int i = threadIdx.x; i < 16 * a.B; i += blockDim.x) {
      const long long o = (long long)(i >> 4) * a.H + nt * 16 + (i & 15);
      if (a.y_f32)
        reinterpret_cast<float*>(a.y)[o] = __int_as_float(0x7FC00000);
      else
        reinterpret_cast<__nv_bfloat16*>(a.y)[o] = __ushort_as_bfloat16((unsigned short)0x7FC0);
    }
}

// ------------------------------------------------------------------ peer all-reduce
// s4: this rank's partial of output tile nt in, the sum over ranks out (exchange.cuh). False if a
// peer's words did not arrive within kPeerWaitNs (s4 is then incomplete).
__device__ __noinline__ bool ar_tile(const FusedArgs& a, int nt, unsigned ep, float4& s4, int lane) {
  return ll_allreduce_tile(a.ar_slots, a.ar_world, a.ar_rank, a.H / 16, nt, a.B, ep, s4, lane, kPeerWaitNs);
}

// ------------------------------------------------------------------ the kernel
// A published w1|w3 segment: kind 1 = tile t of slot s (np items), kind 3 = tile of slot s finished
// by this warp alone (only the slot's count is due).
struct Pend {
  int kind, s, t, np;
};

// TM: phase 1 with CTA-owned tiles (few tiles per CTA); otherwise published segments.
// NTX: the most n-tiles of 4 tokens a slot can need (1 for B <= 4, 2 above); with NTX = 1 the
// two-n-tile code is not compiled in, which keeps the streaming loops small in the instruction cache.
template <int RFMT, bool TM, int NTX>
__global__ void __launch_bounds__(FT, 1) moe_fused_kernel(FusedArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const SmemLayout SL = smem_layout(a.H, a.I_loc, a.B, a.E);
  uint8_t* ring = smem;
  uint8_t* xq = smem + SL.xq;
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem + SL.xs);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + SL.bars);
  uint64_t* hbar = full + NST;
  uint64_t* xbar = full + NST + 1;
  uint64_t* tbar = full + NST + 2;  // [2] a tile's partials written (FW arrivals), by tile parity
  uint64_t* rbar = full + NST + 4;  // [2] a tile's partials reduced (1 arrival), by tile parity
  FPlan& pl = *reinterpret_cast<FPlan*>(smem + SL.plan);
  unsigned* emask = reinterpret_cast<unsigned*>(smem + SL.emask);
  const int lo_off = a.B * a.H + 64;  // lo token rows after the hi rows (opposite bank half)
  const int rp = hq_row_bytes(a.I_loc);
  constexpr float fmtf = RFMT == DSMOE_FMT_FP4 ? kFp4E4m3Scale : 1.0f;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int G = gridDim.x, cta = blockIdx.x;
  const Geo geo = make_geo(a);
  const Span rspan = cta_span(geo.NR, cta, G);
  const int my_router = rspan.e - rspan.s;
  const int nR = my_router > warp ? (my_router - warp + FW - 1) / FW : 0;  // rows rspan.s + warp + FW * k

  if (tid == 0) {
    for (int s = 0; s < NST + 2; ++s) mbar_init(&full[s], 1);  // stage barriers, h barrier, token-row barrier
    mbar_init(&tbar[0], FW);
    mbar_init(&tbar[1], FW);
    mbar_init(&rbar[0], 1);
    mbar_init(&rbar[1], 1);
    pl.abort = 0;
    fence_mbar_init();
  }
  __syncthreads();

  // ---- the warp's item stream: items k < nR are router rows (phase R), the next n1 belong to phase
  // 1 and the last n2 to phase 2 (both known once the plan is). Item k lives in stage (k & 1).
  int kc = 0, ki = 0;  // next item to consume / to issue (warp-uniform)
  int nr = 0, n1 = 0, n2 = 0, N2 = 0, N1 = 0, NR1 = 0;
  // cost of a routed item relative to a shared (FP8) one: FP4 items hold twice the weights
  constexpr int wr = RFMT == DSMOE_FMT_FP4 ? 2 : 1;
  Split sp1{0, 0, 1, 1}, sp2{0, 0, 1, 1};  // phase-1 (published segments) / phase-2 item splits
  int tau0 = 0, ntl = 0;  // phase 1 (TM): this CTA's tiles [tau0, tau0 + ntl)
  Span run1{0, 0}, run2{0, 0};  // phase 1 (published segments) / phase 2 warp runs
  bool planned = false;
  const uint64_t pol_stream = l2_evict_first();
  auto stage_of = [&](int k) { return ring + (size_t)(warp * SPW + (k & 1)) * FSTAGE; };
  auto bar_of = [&](int k) { return &full[warp * SPW + (k & 1)]; };
  TCursor ic1{0, 0};
  Cursor icP{0, 0, 0}, ic2{0, 0, 0};  // issue-side positions of the next phase-1 (TM / segments) / phase-2 item
  // the packed bytes of phase-2 item (slot c.s, n-tile c.t, part c.p)
  auto w2_src = [&](const Cursor& c, const uint8_t*& src, uint32_t& bytes) {
    const W2Item w = {c.s, c.t, c.p};
    if (w.s < nr && RFMT == DSMOE_FMT_FP4) {
      const int c0 = 16 * w.p;
      src = a.r_w2 + (long long)pl.expert[w.s] * a.r_w2_eb + w.nt * geo.tile2r + (long long)c0 * 544;
      bytes = (uint32_t)(min(16, a.I_loc / 64 - c0) * 544);
    } else {
      const uint8_t* tile = w.s < nr ? a.r_w2 + (long long)pl.expert[w.s] * a.r_w2_eb + w.nt * geo.tile2r
                                     : a.s_w2 + w.nt * geo.tile2s;
      const int KC = a.I_loc / 32, c0 = 16 * w.p;
      const int n0 = min(8, KC - c0), n1c = min(8, KC - c0 - 8);
      src = tile + (long long)(2 * w.p) * kFp8W2Item;
      bytes = (uint32_t)(n0 * 512 + 32 + (n0 == 8 && n1c > 0 ? n1c * 512 + 32 : 0));
    }
  };
  auto issue = [&](int k) {  // lane 0: item k's bytes into its stage
    const uint8_t* src;
    uint32_t bytes;
    if (k < nR) {
      const int i = rspan.s + warp + FW * k;
      src = reinterpret_cast<const uint8_t*>(a.wg + (long long)(i >> 2) * a.H + (i & 3) * (a.H / 4));
      bytes = (uint32_t)a.H;
    } else if (k < nR + n1) {
      const uint32_t ib = RFMT == DSMOE_FMT_FP8 ? kFp8W13Item : FCH * 1088;
      if constexpr (TM) {
        const int tau = tau0 + ic1.k;
        if (tau < nr * geo.T) {
          const int sl = tau / geo.T, t = tau - sl * geo.T;
          src = a.r_w13 + (long long)pl.expert[sl] * a.r_w13_eb + t * geo.tile13r + (long long)ic1.p * ib;
          bytes = ib;
        } else {
          src = a.s_w13 + (tau - nr * geo.T) * geo.tile13s + (long long)ic1.p * kFp8W13Item;
          bytes = kFp8W13Item;
        }
      } else {
        if (icP.s < nr) {
          src = a.r_w13 + (long long)pl.expert[icP.s] * a.r_w13_eb + icP.t * geo.tile13r + (long long)icP.p * ib;
          bytes = ib;
        } else {
          src = a.s_w13 + icP.t * geo.tile13s + (long long)icP.p * kFp8W13Item;
          bytes = kFp8W13Item;
        }
      }
    } else {
      w2_src(ic2, src, bytes);
    }
    // The warp's reads of this stage (its previous item) have all completed: each fed an MMA whose
    // result was consumed before this refill, so the copy cannot overtake them.
    mbar_expect_tx(bar_of(k), bytes);
    bulk_g2s_hint(stage_of(k), src, bytes, bar_of(k), pol_stream);
  };
  auto refill = [&]() {  // keep SPW items of the known stream in flight
    const int known = planned ? nR + n1 + n2 : nR;
    while (ki < kc + SPW && ki < known) {
      if (lane == 0) issue(ki);
      if (ki >= nR + n1)
        ic2.next(nr, geo.NT, geo.P2r, geo.P2s);
      else if (ki >= nR) {
        if constexpr (TM)
          ic1.next(geo, nr, tau0, ntl, warp);
        else
          icP.next(nr, geo.T, geo.P13r, geo.P13s);
      }
      ++ki;
    }
  };
  auto wait_full = [&](int k) -> bool {
    if (*(volatile int*)&pl.abort) return false;
    if (!mbar_wait(bar_of(k), (k >> 1) & 1, kWaitNs)) {
      if (lane == 0) {
        atomicOr(a.status, ST_FULL);
        pl.abort = 1;
      }
      return false;
    }
    return true;
  };
  auto drain = [&]() {  // every copy this warp issued lands before the CTA exits
    for (int k = kc; k < ki; ++k) mbar_wait(bar_of(k), (k >> 1) & 1, kWaitNs);
  };
  // bounded grid barrier j (the launch has one, C: j = 0) by thread 0, with the CTA's
  // __syncthreads around it; false = abandon the call. gbase: thread 0's launch base of the arrival
  // counter.
  unsigned long long gbase = 0;
  auto grid_sync = [&](int j) -> bool {
    __syncthreads();
    if (tid == 0 && !pl.abort) {
      grid_arrive(a.gbar);
      if (!grid_wait(a.gbar, gbase + (unsigned long long)(j + 1) * G, a.status)) {
        atomicOr(a.status, ST_GRID);
        pl.abort = 1;
      }
    }
    __syncthreads();
    return !pl.abort;
  };

  // Prologue on constant data only (router rows, shared expert weights). With a programmatic
  // dependent launch it overlaps the previous kernel of the stream, which may still be running.
  refill();  // router rows stream in while the token rows arrive
  // Past this point the previous kernel of the stream has completed and its writes are visible:
  // this call's tokens (often that kernel's output), the workspace, the exchange epoch. The next
  // kernel may be scheduled now; it cannot be resident on an SM before this grid's CTA there exits.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (tid == 0) {
    gbase = grid_base(a.gbar, G);
    pl.rl_epoch = (unsigned)((gbase / (unsigned long long)G) % 0xFFFFFFFFull) + 1u;
    // the peer exchange's epoch of this call: one past the last call's (every CTA reads it here;
    // CTA 0 stores it back after grid barrier C)
    pl.ar_epoch = a.ar_world > 1 ? *(volatile unsigned*)a.ar_ctl + 1u : 0u;
    if (a.B <= FXB) {  // bf16 token rows for the router, one bulk copy
      mbar_expect_tx(xbar, (uint32_t)(a.B * a.H * 2));
      bulk_g2s(xs, a.x, (uint32_t)(a.B * a.H * 2), xbar);
    }
  }
  for (int e = tid; e < a.E; e += FT) emask[e] = 0u;
  // (the finished-tile counts per slot were zeroed at the end of the previous launch)

  if (a.B <= FXB && !mbar_wait(xbar, 0, kWaitNs)) {
    if (tid == 0) {
      atomicOr(a.status, ST_FULL);
      pl.abort = 1;
    }
  }
  __syncthreads();  // pl.rl_epoch

  // ---- phase R: router quarter-rows
  {
    const __nv_bfloat16* xsrc = a.B <= FXB ? xs : a.x;
    while (kc < nR) {
      if (!wait_full(kc)) break;
      const int i = rspan.s + warp + FW * kc;
      router_item(a, stage_of(kc), xsrc, i >> 2, i & 3, lane, pl.rl_epoch);
      __syncwarp();
      ++kc;
      refill();
    }
  }
  // The shared expert's weights do not depend on routing: pull them into L2 while the grid waits for
  // the other CTAs' router partials and plans (each warp a slice; after the router rows, which are
  // on the critical path).
  if (lane == 0) {
    const long long b13 = (long long)geo.T * geo.tile13s, b2 = (long long)geo.NT * geo.tile2s;
    const long long piece = 16384, n13 = (b13 + piece - 1) / piece, n2p = (b2 + piece - 1) / piece;
    for (long long q = (long long)cta * FW + warp; q < n13 + n2p; q += (long long)G * FW) {
      const bool w2p = q >= n13;
      const long long off = (w2p ? q - n13 : q) * piece, tot = w2p ? b2 : b13;
      const uint32_t len = (uint32_t)min(piece, tot - off);
      const uint8_t* src = (w2p ? a.s_w2 : a.s_w13) + off;
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(len) : "memory");
    }
  }
  // token rows -> e4m3 hi / lo while the other CTAs' router partials arrive
  setup_tokens(a, xq, xs, pl, lo_off);
  if (pl.abort) {
    drain();
    poison_y(a);
    return;
  }

  // ---- plan: identical in every CTA. The ring is idle here (phase R consumed, phase 1 not yet
  // issued), so its first bytes hold the scores.
  {
    float* sc_s = reinterpret_cast<float*>(ring);  // [B][E] scores
    float* bi_s = sc_s + a.B * a.E;                // [B][E] scores + selection bias
    const int n = a.B * a.E;
    // every router partial of the launch, polled until both words carry this launch's tag (no grid
    // barrier); two logits per thread per pass, all their loads in flight together
    const unsigned ep = pl.rl_epoch;
    const uint64_t t0 = globaltimer_ns();
    for (int i0 = tid; i0 < n; i0 += 2 * FT) {
      double q[2][4];
      float bias[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int i = i0 + u * FT;
        if (i < n) {
          const int b = i / a.E, e = i - b * a.E;
          const bool vl = a.bias_vl != nullptr && a.image_mask != nullptr && a.image_mask[b] != 0;
          bias[u] = (vl ? a.bias_vl : a.bias)[e];
        }
      }
      unsigned need = 0u;  // bit 4u + c: partial c of logit u still missing
#pragma unroll
      for (int u = 0; u < 2; ++u)
        if (i0 + u * FT < n) need |= 0xFu << (4 * u);
      while (need != 0u) {
        unsigned long long w[2][4][2];
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
          for (int c = 0; c < 4; ++c)
            if ((need >> (4 * u + c)) & 1u) ld_ll2(a.rl + 2 * ((long long)(i0 + u * FT) * 4 + c), w[u][c][0], w[u][c][1]);
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
          for (int c = 0; c < 4; ++c)
            if (((need >> (4 * u + c)) & 1u) && (unsigned)(w[u][c][0] >> 32) == ep && (unsigned)(w[u][c][1] >> 32) == ep) {
              q[u][c] = __longlong_as_double((long long)((w[u][c][0] << 32) | (w[u][c][1] & 0xFFFFFFFFull)));
              need &= ~(1u << (4 * u + c));
            }
        if (need != 0u && (ld_relaxed_u32(a.status) != 0u || globaltimer_ns() - t0 > kWaitNs)) {
          atomicOr(a.status, ST_GRID);
          pl.abort = 1;
          break;
        }
      }
      if (need != 0u) break;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int i = i0 + u * FT;
        if (i < n) {
          const double l = ((q[u][0] + q[u][1]) + q[u][2]) + q[u][3];
          const float s = fscore(__double2float_rn(l), a.score_func);
          sc_s[i] = s;
          bi_s[i] = s + bias[u];
        }
      }
    }
    __syncthreads();
    if (pl.abort) {
      drain();
      poison_y(a);
      return;
    }
    if (cta == 0 && a.scores)
      for (int i = tid; i < n; i += FT) a.scores[i] = sc_s[i];
    // top-k of token b (warp b): the token's biased scores in registers (expert lane + 32 j) as
    // order-preserving keys, then k rounds of (lane-local best, warp max, lowest index holding it),
    // the winner's lane dropping it; ties -> lower index
    for (int b = warp; b < a.B; b += FW) {
      float tot = 0.f;
      if (a.E <= 32 * FKJ)
        topk_token<FKJ>(bi_s + b * a.E, sc_s + b * a.E, a.E, a.topk, lane, pl.sel[b], pl.selw[b], tot);
      else
        topk_token<FEMAX / 32>(bi_s + b * a.E, sc_s + b * a.E, a.E, a.topk, lane, pl.sel[b], pl.selw[b], tot);
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
    __syncthreads();
    if (a.B == 1) {
      // one token: its k (distinct) picks are the slots, in expert order (rank = picks below it)
      if (warp == 0 && lane < a.topk) {
        const int e = pl.sel[0][lane];
        int rk = 0;
        for (int r = 0; r < a.topk; ++r) rk += pl.sel[0][r] < e ? 1 : 0;
        pl.expert[rk] = e;
        pl.ntok[rk] = 1;
        for (int c = 0; c < 8; ++c) {
          pl.tok[rk][c] = 0;
          pl.wt[rk][c] = c == 0 ? pl.selw[0][lane] : 0.f;
          pl.col_of[rk][c] = c == 0 ? (signed char)0 : (signed char)-1;
        }
      }
      if (tid == 0) {
        const int sh = a.topk;  // the shared expert's slot
        pl.n_routed = a.topk;
        pl.expert[sh] = a.E;
        pl.ntok[sh] = 1;
        for (int c = 0; c < 8; ++c) {
          pl.tok[sh][c] = 0;
          pl.wt[sh][c] = 1.0f;
          pl.col_of[sh][c] = c == 0 ? (signed char)0 : (signed char)-1;
        }
      }
      __syncthreads();
    } else {
    for (int i = tid; i < a.B * a.topk; i += FT) atomicOr(&emask[pl.sel[i / a.topk][i % a.topk]], 1u << (i / a.topk));
    __syncthreads();
    // slots in expert order: block-wide compaction of the experts with picks
    int base = 0;
    for (int e0 = 0; e0 < a.E; e0 += FT) {
      const int e = e0 + tid;
      const unsigned m = e < a.E ? emask[e] : 0u;
      const unsigned bal = __ballot_sync(0xffffffffu, m != 0u);
      if (lane == 0) pl.wcnt[warp] = __popc(bal);
      __syncthreads();
      int off = base, total = 0;
      for (int w = 0; w < FW; ++w) {
        if (w < warp) off += pl.wcnt[w];
        total += pl.wcnt[w];
      }
      off += __popc(bal & ((1u << lane) - 1u));
      if (m != 0u) {
        pl.expert[off] = e;
        pl.ntok[off] = __popc(m);
        int cnt = 0;
        for (int b = 0; b < FMAXB; ++b) pl.col_of[off][b] = -1;
        for (int b = 0; b < a.B; ++b) {
          if (m & (1u << b)) {
            float w = 0.f;
            for (int r = 0; r < a.topk; ++r)
              if (pl.sel[b][r] == e) w = pl.selw[b][r];
            pl.tok[off][cnt] = b;
            pl.wt[off][cnt] = w;
            pl.col_of[off][b] = (signed char)cnt;
            ++cnt;
          }
        }
        for (; cnt < 8; ++cnt) {
          pl.tok[off][cnt] = pl.tok[off][0];
          pl.wt[off][cnt] = 0.f;
        }
      }
      base += total;
      __syncthreads();
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
    __syncthreads();
    }
  }



  // ---- the rest of the stream is known. Phase 1: this CTA's w1|w3 tiles (routed slots' tiles,
  // then the shared expert's as slot nr), each tile's parts split over the warps; phase 2: w2 items.
  nr = pl.n_routed;
  if constexpr (TM) {
    const Span ts = cta_span((nr + 1) * geo.T, cta, G);
    tau0 = ts.s;
    ntl = ts.e - ts.s;
    n1 = 0;
    for (int k = 0; k < ntl; ++k) {
      const int P = tile_nparts(geo, nr, tau0 + k), j = run_of(warp, k);
      n1 += P * (j + 1) / FW - P * j / FW;
    }
    ic1.start(geo, nr, tau0, ntl, warp);
  } else {  // items (slot, tile, part): routed slots' tiles of P13r items, then the shared slot's
    NR1 = nr * geo.T * geo.P13r;
    N1 = NR1 + geo.T * geo.P13s;
    sp1 = Split{N1, NR1, wr, 1};
    run1 = warp_run(sp1.span(cta, G), warp);
    n1 = run1.e - run1.s;
    icP = cursor1(geo, nr, NR1, run1.s);
  }
  N2 = nr * geo.NT * geo.P2r + geo.NT * geo.P2s;
  sp2 = Split{N2, nr * geo.NT * geo.P2r, wr, 1};
  run2 = warp_run(sp2.span(cta, G), warp);
  n2 = run2.e - run2.s;
  ic2 = cursor2(geo, nr, run2.s);
  planned = true;
  refill();

  // the lane's token row (B column g = lane / 4) of n-tiles 0 and 1, for a slot's token list
  auto token_rows = [&](const uint8_t** xr, const int* toks, int ntok) {
#pragma unroll
    for (int j = 0; j < 2; ++j)
      xr[j] = xq + (size_t)toks[min(4 * j + (lane >> 3), ntok - 1)] * a.H + ((lane >> 2) & 1) * lo_off + (lane & 3) * 16;
  };

  if constexpr (TM) {
  // ---- phase 1: w1|w3 of this CTA's tiles. Each warp accumulates its run of a tile's parts, writes
  // its partial (8 floats per lane) to the CTA's slot of the scratch and arrives on the tile's
  // barrier; warp k % FW sums the FW partials in warp order (deterministic), applies clamp / SiLU / up -> h
  // rows, and counts the tile for its slot. Partial slots alternate by tile parity: a warp writes
  // tile k's only after tile k - 2's reduction has read them.
  {
    float* gp = a.p13 + (size_t)cta * 2 * FW * 256;  // [parity][warp][32 lanes][8]
    float acc1[2][4], acc3[2][4];
    const uint8_t* xr[2] = {xq, xq};
    for (int k = 0; k < ntl && !pl.abort; ++k) {
      const int tau = tau0 + k;
      const int sl = tau < nr * geo.T ? tau / geo.T : nr, t = tau - sl * geo.T;
      const int sidx = sl < nr ? sl : a.sh_idx;
      const int P = tile_nparts(geo, nr, tau), j = run_of(warp, k), pb = P * j / FW, pe = P * (j + 1) / FW;
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc1[j][q] = acc3[j][q] = 0.f;
      token_rows(xr, pl.tok[sl], pl.ntok[sl]);
      const bool two = NTX == 2 && pl.ntok[sl] > 4;
      for (int p = pb; p < pe; ++p) {
        if (!wait_full(kc)) break;
        const uint8_t* stage = stage_of(kc);
        if (sl < nr) {
          if (two)
            w13_accum<RFMT, 2>(stage, xr, p, lane, acc1, acc3);
          else
            w13_accum<RFMT, 1>(stage, xr, p, lane, acc1, acc3);
        } else {
          if (two)
            w13_accum<DSMOE_FMT_FP8, 2>(stage, xr, p, lane, acc1, acc3);
          else
            w13_accum<DSMOE_FMT_FP8, 1>(stage, xr, p, lane, acc1, acc3);
        }
        __syncwarp();
        ++kc;
        refill();
      }
      if (pl.abort) break;
      float s8[8];
      w13_combine(acc1, acc3, s8);
      float* mine = gp + ((size_t)((k & 1) * FW + warp) * 32 + lane) * 8;
      if (k >= 2 && !mbar_wait(&rbar[k & 1], ((k - 2) >> 1) & 1, kWaitNs)) {
        if (lane == 0) {
          atomicOr(a.status, ST_SLOT);
          pl.abort = 1;
        }
        break;
      }
      *reinterpret_cast<float4*>(mine) = make_float4(s8[0], s8[1], s8[2], s8[3]);
      *reinterpret_cast<float4*>(mine + 4) = make_float4(s8[4], s8[5], s8[6], s8[7]);
      __syncwarp();
      if (lane == 0) mbar_arrive(&tbar[k & 1]);
      if (warp == k % FW) {
        if (!mbar_wait(&tbar[k & 1], (k >> 1) & 1, kWaitNs)) {
          if (lane == 0) {
            atomicOr(a.status, ST_SLOT);
            pl.abort = 1;
          }
          break;
        }
        float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int w = 0; w < FW; ++w) {  // warp order
          const float* src = gp + ((size_t)((k & 1) * FW + w) * 32 + lane) * 8;
          const float4 u0 = *reinterpret_cast<const float4*>(src), u1 = *reinterpret_cast<const float4*>(src + 4);
          v[0] += u0.x;
          v[1] += u0.y;
          v[2] += u0.z;
          v[3] += u0.w;
          v[4] += u1.x;
          v[5] += u1.y;
          v[6] += u1.z;
          v[7] += u1.w;
        }
        w13_epilogue(a, pl, sidx, t, v, pl.ntok[sl], pl.tok[sl], sl < nr ? fmtf : 1.0f, lane);
        fence_acq_rel_gpu();
        __syncwarp();
        if (lane == 0) {
          atomicAdd(a.slot_done + sidx, 1u);
          mbar_arrive(&rbar[k & 1]);
        }
      }
    }
  }
  } else {
  // phase-1 tile (slot s, tile t): its first item and its part count
  auto tile_first = [&](int s, int t) { return s < nr ? (s * geo.T + t) * geo.P13r : NR1 + t * geo.P13s; };
  auto tile_parts = [&](int s) { return s < nr ? geo.P13r : geo.P13s; };

  // ---- published segments: one fence for the batch, one counter per tile, one acquire fence if
  // this warp finished any; the last contributor applies the epilogue and counts the slot's tile
  Pend pend[NPEND];
  int npend = 0;
  auto publish = [&]() {
    if (npend == 0) return;
    fence_acq_rel_gpu();
    __syncwarp();
    // lane i counts pending segment i's items on its tile, all lanes at once (one round trip)
    unsigned* mycnt = nullptr;
    int mynp = 0, myparts = 0;
    for (int i = 0; i < npend; ++i)
      if (i == lane && pend[i].kind != 3) {
        mycnt = a.cnt13 + (pend[i].s < nr ? pend[i].s : a.sh_idx) * geo.T + pend[i].t;
        mynp = pend[i].np;
        myparts = tile_parts(pend[i].s);
      }
    unsigned old = 0;
    if (mycnt) old = atomicAdd(mycnt, (unsigned)mynp);
    // bit i: this warp completed pending segment i's tile
    const unsigned last = __ballot_sync(0xffffffffu, mycnt != nullptr && (int)old + mynp == myparts);
    if (last) fence_acq_rel_gpu();
    for (int i = 0; i < npend; ++i) {
      if (!((last >> i) & 1u)) continue;
      const Pend e = pend[i];
      const int sidx = e.s < nr ? e.s : a.sh_idx;
      float s8[8];
      w13_reduce(a, geo, sidx, e.t, tile_first(e.s, e.t), tile_parts(e.s), sp1, lane, s8);
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = s8[j];
      w13_epilogue(a, pl, sidx, e.t, v, pl.ntok[e.s], pl.tok[e.s], e.s < nr ? fmtf : 1.0f, lane);
      if (lane == 0) a.cnt13[sidx * geo.T + e.t] = 0u;
    }
    fence_acq_rel_gpu();
    __syncwarp();
    if (lane == 0)
      for (int i = 0; i < npend; ++i)
        if (pend[i].kind == 3 || ((last >> i) & 1u)) atomicAdd(a.slot_done + (pend[i].s < nr ? pend[i].s : a.sh_idx), 1u);
    npend = 0;
  };
  auto add_pend = [&](int kind, int s, int t, int np) {
    pend[npend++] = {kind, s, t, np};
    if (npend == NPEND) publish();
  };

  // ---- phase 1: w1|w3 of every slot
  {
    int cur_s = -1, cur_t = -1, seg_first = 0, seg_np = 0;
    float acc1[2][4], acc3[2][4];
    const uint8_t* xr[2] = {xq, xq};
    auto end_seg = [&]() {
      const int sidx = cur_s < nr ? cur_s : a.sh_idx;
      float s8[8];
      w13_combine(acc1, acc3, s8);
      if (seg_np == tile_parts(cur_s)) {
        w13_epilogue(a, pl, sidx, cur_t, s8, pl.ntok[cur_s], pl.tok[cur_s], cur_s < nr ? fmtf : 1.0f, lane);
        add_pend(3, cur_s, cur_t, 0);
      } else {
        float* dst = p13_slot(a, geo, sidx, cur_t, seg_first - tile_first(cur_s, cur_t), lane);
        *reinterpret_cast<float4*>(dst) = make_float4(s8[0], s8[1], s8[2], s8[3]);
        *reinterpret_cast<float4*>(dst + 4) = make_float4(s8[4], s8[5], s8[6], s8[7]);
        add_pend(1, cur_s, cur_t, seg_np);
      }
    };
    Cursor cc = cursor1(geo, nr, NR1, run1.s);
    while (kc < nR + n1) {
      if (!wait_full(kc)) break;
      const int i = run1.s + (kc - nR);
      const int s = cc.s, t = cc.t, p = cc.p;
      cc.next(nr, geo.T, geo.P13r, geo.P13s);
      if (s != cur_s || t != cur_t) {
        if (cur_s >= 0) end_seg();
        cur_s = s;
        cur_t = t;
        seg_first = i;
        seg_np = 0;
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int q = 0; q < 4; ++q) acc1[j][q] = acc3[j][q] = 0.f;
        token_rows(xr, pl.tok[s], pl.ntok[s]);
      }
      const uint8_t* stage = stage_of(kc);
      const bool two = NTX == 2 && pl.ntok[s] > 4;
      if (s < nr) {
        if (two)
          w13_accum<RFMT, 2>(stage, xr, p, lane, acc1, acc3);
        else
          w13_accum<RFMT, 1>(stage, xr, p, lane, acc1, acc3);
      } else {
        if (two)
          w13_accum<DSMOE_FMT_FP8, 2>(stage, xr, p, lane, acc1, acc3);
        else
          w13_accum<DSMOE_FMT_FP8, 1>(stage, xr, p, lane, acc1, acc3);
      }
      ++seg_np;
      __syncwarp();
      ++kc;
      refill();
    }
    if (cur_s >= 0 && !pl.abort) end_seg();
    if (!pl.abort) publish();
  }
  }

  // ---- phase 2 set-up: the h rows of the (at most FHSLOTS) slots of this CTA's span, once their
  // w1|w3 tiles are all finished, into the token-row region (free after phase 1)
  const Span span2 = sp2.span(cta, G);
  int sA = 0, sB = -1;
  if (span2.e > span2.s) {
    sA = w2_item(geo, nr, span2.s).s;
    sB = w2_item(geo, nr, span2.e - 1).s;
  }
  __syncthreads();
  if (tid == 0 && sB >= sA && !pl.abort) {
    bool ok = sB - sA + 1 <= FHSLOTS;
    if (!ok) atomicOr(a.status, ST_SLOT);
    const uint64_t t0 = globaltimer_ns();
    for (int s = sA; s <= sB && ok; ++s) {
      const unsigned* cnt = a.slot_done + (s < nr ? s : a.sh_idx);
      while (ld_relaxed_u32(cnt) < (unsigned)geo.T) {
        if (ld_relaxed_u32(a.status) != 0u || globaltimer_ns() - t0 > kWaitNs) {
          atomicOr(a.status, ST_SLOT);
          ok = false;
          break;
        }
      }
    }
    if (ok) {
      fence_acq_rel_gpu();
      asm volatile("fence.proxy.async.global;" ::: "memory");
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      uint32_t total = 0;
      for (int s = sA; s <= sB; ++s) total += 2u * pl.ntok[s] * rp;
      mbar_expect_tx(hbar, total);
      for (int s = sA; s <= sB; ++s) {
        const int sidx = s < nr ? s : a.sh_idx, nt = pl.ntok[s];
        uint8_t* dst = xq + (size_t)(s - sA) * SL.hs_stride;
        bulk_g2s(dst, a.hq + hq_row(a.I_loc, sidx, 0, 0), (uint32_t)(nt * rp), hbar);
        bulk_g2s(dst + nt * rp + 64, a.hq + hq_row(a.I_loc, sidx, 1, 0), (uint32_t)(nt * rp), hbar);
      }
    } else {
      pl.abort = 1;
    }
  }
  __syncthreads();
  if (pl.abort) {
    drain();
    poison_y(a);
    return;
  }
  if (sB >= sA && !mbar_wait(hbar, 0, kWaitNs)) {
    if (lane == 0) {
      atomicOr(a.status, ST_SLOT);
      pl.abort = 1;
    }
  }

  // ---- phase 2: w2; each (slot, n-tile) segment folded into token columns and written as a partial
  {
    int cur_s = -1, cur_nt = -1, seg_first = 0, seg_np = 0;
    const uint8_t* hbase = xq;
    float tot[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int q = 0; q < 4; ++q) tot[j][q] = 0.f;
    auto end_seg = [&]() {
      float out[4] = {0.f, 0.f, 0.f, 0.f};
      const float fs = (cur_s < nr && RFMT == DSMOE_FMT_FP4 ? kFp4E4m3Scale : 1.0f) / kHScale;
      w2_fold(a, pl, cur_s, fs, tot, lane, out);
      const int rel = seg_first - w2_range_start(geo, nr, cur_s, cur_nt);
      *reinterpret_cast<float4*>(p2_slot(a, cur_nt, cur_s, rel, lane)) = make_float4(out[0], out[1], out[2], out[3]);
      for (int q = 1; q < seg_np; ++q)
        *reinterpret_cast<float4*>(p2_slot(a, cur_nt, cur_s, rel + q, lane)) = make_float4(0.f, 0.f, 0.f, 0.f);
    };
    Cursor cc = cursor2(geo, nr, run2.s);
    while (kc < nR + n1 + n2) {
      if (!wait_full(kc)) break;
      const int i = run2.s + (kc - nR - n1);
      const W2Item w = {cc.s, cc.t, cc.p};
      cc.next(nr, geo.NT, geo.P2r, geo.P2s);
      if (w.s != cur_s || w.nt != cur_nt) {
        if (cur_s >= 0) end_seg();
        cur_s = w.s;
        cur_nt = w.nt;
        seg_first = i;
        seg_np = 0;
        hbase = xq + (size_t)(w.s - sA) * SL.hs_stride;
      }
      ++seg_np;
      const uint8_t* stage = stage_of(kc);
      const int ntok = pl.ntok[w.s];
      if (w.s < nr) {
        if (NTX == 2 && ntok > 4)
          w2_accum<RFMT, 2>(a, stage, hbase, rp, ntok, w.p, lane, tot);
        else
          w2_accum<RFMT, 1>(a, stage, hbase, rp, ntok, w.p, lane, tot);
      } else {
        if (NTX == 2 && ntok > 4)
          w2_accum<DSMOE_FMT_FP8, 2>(a, stage, hbase, rp, ntok, w.p, lane, tot);
        else
          w2_accum<DSMOE_FMT_FP8, 1>(a, stage, hbase, rp, ntok, w.p, lane, tot);
      }
      __syncwarp();
      ++kc;
      refill();
    }
    if (cur_s >= 0 && !pl.abort) end_seg();
  }
  drain();
  // ---- grid barrier C, then each CTA finishes its 16-row output tiles nt = cta + G * j: the warps
  // split each tile's positions into fixed chunks summed in order, and the chunk sums are added in
  // chunk order -> y (deterministic)
  if (!grid_sync(0)) {
    poison_y(a);
    return;
  }
  // every CTA is past its phase-2 waits on the finished-tile counts: zero them for the next launch
  // (which starts after this grid completes), and store the exchange epoch every CTA read at start
  if (tid == 0) {
    for (int i = cta; i < a.slots; i += G) a.slot_done[i] = 0u;
    if (cta == 0 && a.ar_world > 1)
      asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(a.ar_ctl), "r"(pl.ar_epoch) : "memory");
  }
  const int nn = cta < geo.NT ? (geo.NT - 1 - cta) / G + 1 : 0;
  if (nn > 0) {
    const int P = nr * geo.P2r + geo.P2s;
    const int j = warp % nn, ci = warp / nn, nw = (FW - j + nn - 1) / nn;
    const float4 part = w2_chunk_sum(a, geo, nr, cta + G * j, P * ci / nw, P * (ci + 1) / nw, lane);
    float4* red = reinterpret_cast<float4*>(ring);  // idle after phase 2
    red[warp * 32 + lane] = part;
    __syncthreads();
    if (warp < nn) {
      float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int c = 0; c < nw; ++c) {
        const float4 v = red[(c * nn + warp) * 32 + lane];
        s4.x += v.x;
        s4.y += v.y;
        s4.z += v.z;
        s4.w += v.w;
      }
      if (a.ar_world > 1 && !ar_tile(a, cta + G * warp, pl.ar_epoch, s4, lane)) {
        if (lane == 0) atomicOr(a.status, ST_PEER);
        s4 = make_float4(__int_as_float(0x7FC00000), __int_as_float(0x7FC00000), __int_as_float(0x7FC00000),
                         __int_as_float(0x7FC00000));
      }
      w2_store_y(a, cta + G * warp, s4, lane);
    }
  }
}

// ------------------------------------------------------------------ host side
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
  f.p13max = (H / 32) / FCH;                // FP8 parts per tile bound both formats
  f.p2max = (I_loc + FK2_8 - 1) / FK2_8;    // FP8 w2 items per (slot, n-tile) bound both formats
  size_t o = 0;
  f.gbar = o; o += al2(8);
  f.status = o; o += al2(4);
  f.cnt2 = o; o += al2((size_t)NT * 4);
  f.cnt13 = o; o += al2((size_t)f.slots * T * 4);
  f.slot_done = o; o += al2((size_t)f.slots * 4);
  f.rl = o; o += al2((size_t)B * E * 4 * 16);
  // w1|w3 partials: the larger of the published-segment layout [slots][T][p13max][32][8] and the
  // CTA-owned-tile layout [CTA][2][FW][32][8]
  const size_t p13_seg = (size_t)f.slots * T * f.p13max * 32 * 8 * 4, p13_tm = (size_t)kMaxCtas * 2 * FW * 32 * 8 * 4;
  f.p13 = o; o += al2(p13_seg > p13_tm ? p13_seg : p13_tm);
  f.p2 = o; o += al2((size_t)NT * f.slots * f.p2max * 32 * 4 * 4);
  f.hq = o; o += al2((size_t)f.slots * hq_slot_bytes(I_loc));
  f.total = o;
  return f;
}

// Per-device constants, looked up once (attribute queries cost microseconds per call).
struct DevInfo {
  int sms = 0, optin = 0;
  bool attr_set[8] = {false, false, false, false, false, false, false, false};
  int pdl = -1;  // programmatic dependent launch with the cooperative attribute: -1 untested, 0 no, 1 yes
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

size_t fused_smem_bytes(int H, int I_loc, int B, int E) { return smem_layout(H, I_loc, B, E).total; }

// Geometry the persistent kernel takes: at most 8 tokens and 1024 experts, whole 256-K w1|w3 items,
// a router quarter-row that fits a stage, and phase-2 CTA spans that touch at most FHSLOTS slots.
bool fused_supported(const dsmoe_layer_t* L, int B) {
  if (B < 1 || B > FMAXB || L->n_experts > FEMAX || L->hidden % 512 != 0 || L->hidden > FSTAGE) return false;
  const DevInfo& d = dev_info();
  if (d.sms > kMaxCtas) return false;
  if (fused_smem_bytes(L->hidden, L->inter_local, B, L->n_experts) > (size_t)d.optin) return false;
  const int NT = L->hidden / 16, I = L->inter_local;
  const int P2s = (I + FK2_8 - 1) / FK2_8;
  const int P2r = L->routed.fmt == DSMOE_FMT_FP8 ? P2s : (I + FK2_4 - 1) / FK2_4;
  const long long n2max = (long long)B * L->topk * NT * P2r + (long long)NT * P2s;
  // the longest phase-2 CTA span (items split by cost, routed FP4 items counting twice)
  const long long c2 = (L->routed.fmt == DSMOE_FMT_FP4 ? 2 : 1) * (long long)B * L->topk * NT * P2r + (long long)NT * P2s;
  const long long span = (c2 + d.sms - 1) / d.sms + 1;
  const long long T = I / 16, n1max = (long long)(B * L->topk + 1) * T * ((L->hidden / 32) / FCH);
  const long long nmax = n1max > n2max ? n1max : n2max;
  if (nmax * d.sms >= (1LL << 31) || 4LL * L->n_experts * d.sms >= (1LL << 31)) return false;
  return span <= (long long)NT * (P2r < P2s ? P2r : P2s) + 1;
}

int launch_fused(const dsmoe_layer_t* L, const void* x, int B, const uint8_t* image_mask, void* y, int y_dtype,
                 int64_t* idx, float* wt, float* scores, uint8_t* ws, cudaStream_t st, void* const* events,
                 const PeerExchange* px) {
  DevInfo& d = dev_info();
  const int optin = d.optin, sms = d.sms;
  const size_t smem = fused_smem_bytes(L->hidden, L->inter_local, B, L->n_experts);
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
  a.rl = (unsigned long long*)(ws + f.rl);
  a.p13 = (float*)(ws + f.p13);
  a.p2 = (float*)(ws + f.p2);
  a.hq = ws + f.hq;
  a.cnt13 = (unsigned*)(ws + f.cnt13);
  a.cnt2 = (unsigned*)(ws + f.cnt2);
  a.slot_done = (unsigned*)(ws + f.slot_done);
  a.gbar = (unsigned long long*)(ws + f.gbar);
  a.status = (unsigned*)(ws + f.status);
  a.sh_idx = FMAXB * L->topk;
  a.slots = f.slots;
  a.p13max = f.p13max;
  a.p2max = f.p2max;
  if (px && px->world > 1) {
    DSMOE_REQUIRE(px->hidden == L->hidden && px->world <= kMaxWorld && px->rank >= 0 && px->rank < px->world,
                  DSMOE_ERR_ARG, "fused: exchange for hidden %d, world %d, rank %d", px->hidden, px->world, px->rank);
    a.ar_world = px->world;
    a.ar_rank = px->rank;
    a.ar_ctl = px->ctl;
    for (int q = 0; q < px->world; ++q) {
      DSMOE_REQUIRE(px->slots[q], DSMOE_ERR_ARG, "fused: exchange slots of rank %d not mapped", q);
      a.ar_slots[q] = px->slots[q];
    }
  }

  int fi = L->routed.fmt == DSMOE_FMT_FP8 ? 0 : 1;
  // Phase 1 with CTA-owned tiles when the step has at most about two w1|w3 tiles per CTA (small
  // intermediate slices: tensor parallelism over 4-8 GPUs); published segments otherwise.
  const bool tm = (long long)(B * L->topk + 1) * (L->inter_local / 16) <= 2LL * sms;
  const bool b4 = B <= 4;
  void (*kern)(FusedArgs) =
      fi == 0 ? (tm ? (b4 ? moe_fused_kernel<DSMOE_FMT_FP8, true, 1> : moe_fused_kernel<DSMOE_FMT_FP8, true, 2>)
                    : (b4 ? moe_fused_kernel<DSMOE_FMT_FP8, false, 1> : moe_fused_kernel<DSMOE_FMT_FP8, false, 2>))
              : (tm ? (b4 ? moe_fused_kernel<DSMOE_FMT_FP4, true, 1> : moe_fused_kernel<DSMOE_FMT_FP4, true, 2>)
                    : (b4 ? moe_fused_kernel<DSMOE_FMT_FP4, false, 1> : moe_fused_kernel<DSMOE_FMT_FP4, false, 2>));
  fi += (tm ? 2 : 0) + (b4 ? 4 : 0);
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
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  // Programmatic dependent launch: the kernel's prologue overlaps the tail of the previous kernel
  // in the stream. Tried on the first call outside stream capture; a refusal turns it off.
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (d.pdl < 0) cudaStreamIsCapturing(st, &cap);
  const bool try_pdl = d.pdl == 1 || (d.pdl < 0 && cap == cudaStreamCaptureStatusNone);
  cfg.numAttrs = try_pdl ? 2 : 1;
  if (events) {
    cudaEventRecord((cudaEvent_t)events[0], st);
    cudaEventRecord((cudaEvent_t)events[1], st);
    cudaEventRecord((cudaEvent_t)events[2], st);
  }
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
  if (try_pdl && d.pdl < 0) {
    if (e == cudaSuccess) {
      d.pdl = 1;
    } else {  // not accepted with the cooperative attribute here: launch without it from now on
      cudaGetLastError();
      d.pdl = 0;
      cfg.numAttrs = 1;
      e = cudaLaunchKernelEx(&cfg, kern, a);
    }
  }
  if (events) cudaEventRecord((cudaEvent_t)events[3], st);
  if (e != cudaSuccess) {
    set_error("fused launch: %s", cudaGetErrorString(e));
    cudaGetLastError();
    return DSMOE_ERR_CUDA;
  }
  return DSMOE_OK;
}

}  // namespace dsmoe
