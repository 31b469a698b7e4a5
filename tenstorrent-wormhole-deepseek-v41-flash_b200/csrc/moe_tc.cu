// One persistent tcgen05 kernel per MoE layer for decode batches of 1..8 tokens, on the TC store
// (tcstore.cuh: checkpoint row-major weights, tiled and swizzled by the TMA tensor engine).
//
// Replaces, per decode token and MoE layer, the reference's device router GEMV + host top-k +
// host->device control write + SlotCat gather + w1/w3/shared matmuls + Q20 SwiGLU + w2 matmuls +
// all_gather/sum all-reduce (dsv41/tt/model.py:400-442; dsv41/tt/moe.py:108-180;
// dsv41/kernels/slot_cat.cpp; dsv41/tt/attn.py:19-21) with one launch that streams every weight
// byte of the step once.
//
// Each CTA (one per SM) runs a warp-specialised pipeline over a ring of shared-memory stages, one
// 128-K block of one 128-row weight tile per stage:
//   warp 0      TMA producer: cp.async.bulk.tensor loads of the weight tile (FP8 bytes as stored;
//               FP4 widened by the TMA to the padded e2m1 form the tensor core reads) and the
//               tile's scales, L2 evict-first.
//   warp 1      MMA issuer: tcgen05.mma M 128, N 16 (columns 0..7: e4m3 "hi" parts of the 8
//               token slots, 8..15: their "lo" parts, x ~ hi + lo / 16), K 32 per instruction,
//               accumulators in tensor memory. FP8: kind::f8f6f4, one accumulator per 128-K scale
//               block (the non-MX fp32 block scales are applied by the epilogue); FP4:
//               kind::mxf8f6f4.block_scale with A = e2m1 and the checkpoint's e8m0 scales in
//               tensor memory, so the tensor core applies the 32-K group scales itself.
//   warp 2      phase-2 operand producer: copies each w2 stage's B tile (the slot's SwiGLU output h
//               as e4m3 hi / lo rows) once every w1|w3 tile of that slot is finished, grid-wide.
//   warp 3      finisher: sums a tile's ordered partials once its last contribution lands
//               (w1|w3 tile: clamp / SiLU / up -> h; w2 output tile: routed + shared -> y, then
//               the NVLink peer all-reduce at N > 1).
//   warps 4-7   epilogue: tcgen05.ld of the accumulators (one TMEM lane quadrant each), block
//               scales, routing weights, ordered partials; FP4 scale factors into tensor memory.
// Before the pipeline roles start, warps 1-7 compute the router (fp64-exact logits, tagged
// partials shared through global memory), convert the tokens to the MMA's B tile and plan the slots
// (experts chosen by any token, in expert order, then the shared expert). The producer streams the
// shared expert's w1|w3 (routing-independent) from the first cycle, while the router runs.
//
// Work split: four flat sequences of stages -- shared w1|w3, routed w1|w3 (slot, 64-row tile, K
// block), shared w2, routed w2 (slot, 128-row output tile, K block) -- each cut into contiguous
// per-CTA ranges ("stream-K"). A run of one CTA inside one tile is a unit: its result is one
// partial, stored at the CTA's contributor index within the tile, and the tile's last contribution
// (a launch-tagged counter) hands the tile to that CTA's finisher, which sums the partials in
// contributor order: results are deterministic and independent of timing. Counters carry the
// launch number in their high half, so they never need resetting; there is no grid barrier.
// Every wait is bounded (%globaltimer); on expiry the kernel sets a status bit, stops, lets its
// copies land and writes NaN into its share of y.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "exchange.cuh"
#include "tcstore.cuh"

namespace dsmoe {
namespace tc {

constexpr int NW = 8, NT = NW * 32;
constexpr int MAXB = 8;                  // tokens per call
constexpr int MAXK = DSMOE_MAX_TOPK;
constexpr int MAXSLOT = MAXB * MAXK + 1;  // routed slots + the shared expert
constexpr int MAXE = 1024;
constexpr int MAXC = 6;                  // contributors (CTAs) per tile: bounds the per-CTA range length
constexpr int SA = 16384;                // stage A: 128 rows x 128 K (one byte per element in shared memory)
constexpr int SB = 2048;                 // stage B (w2 phase): 16 rows x 128 K e4m3
constexpr int STAGE = SA + SB + 1024;    // + 1 KB for the stage's scales (FP4 512 B, FP8 16 B)
constexpr int NACC8 = 16;                // FP8 block accumulators (16 TMEM columns each)
constexpr int kDepth8 = 6;               // FP8 stages (16 KB) in flight per CTA
// Tensor memory columns: FP8 block accumulators [0, 256), FP4 unit accumulators [2 parities][2 issuers]
// at [256, 320), FP4 A scale factors 4 per ring slot from 320, B scale factors at 416.
constexpr uint32_t TM_ACC4 = 256, TM_SFA = 320, TM_SFB = 416, TM_COLS = 512;
constexpr int MAXS = 20;                 // ring stages (TM_SFA + 4 MAXS <= TM_SFB)
constexpr int NISS = 2;                  // MMA issuing threads (lane 0 of warp 1 and, at N = 1, of warp 3)
constexpr int QCAP = 64;                 // finisher job queue
constexpr uint64_t kWait = 1000000000ull;
constexpr uint64_t kPeerWait = 5000000000ull;

enum : unsigned { ST_MBAR = 1u, ST_CNT = 2u, ST_PLAN = 4u, ST_PEER = 16u };

struct TcArgs {
  CUtensorMap tm_r13, tm_r2, tm_s13, tm_s2;  // routed / shared w1|w3 (4-D) and w2 (3-D) tensor maps
  int H, I_loc, row0, E, B, topk, score_func;
  float route_scale;
  int r_fmt;
  int P1, KB1, KB2, MT2, S, slot_cap;
  const float* wg;
  const float* bias;
  const float* bias_vl;
  const uint8_t* image_mask;
  const __nv_bfloat16* x;
  const uint8_t* r13;  // routed expert blocks (scale tables after the weights)
  const uint8_t* r2;
  long long r_eb13, r_eb2, r_d13, r_d2;
  const uint8_t* s13;  // shared expert (FP8)
  const uint8_t* s2;
  long long s_d13, s_d2;
  void* y;
  int y_f32;
  int64_t* idx;
  float* wt;
  float* scores;
  // workspace
  unsigned long long* gbar;
  unsigned* status;
  unsigned long long* rl;     // [8][E][4] router quarter-row partials, two tagged words each
  // Counters, one set per launch parity (the set of launch tag t is cnt + (t & 1) cnt_words; the set
  // of the next launch is zeroed while this one runs): [slot_cap][P1] stage counts of w1|w3 tiles,
  // [MT2] stage counts of w2 output tiles, [slot_cap] finished w1|w3 tiles per slot.
  unsigned long long* cnt;
  int cnt_words;
  float* p13;                 // [slot_cap][P1][MAXC][128][8]
  float* p2;                  // [MT2][slot_cap][MAXC][128][8]
  uint8_t* hb;                // [slot_cap][KB2][2048] h as the w2 B tile (e4m3 hi / lo, SW128)
  int ar_world, ar_rank;
  unsigned* ar_ctl;
  unsigned long long* ar_slots[kMaxWorld];
};


// ------------------------------------------------------------------ stream-K split of a sequence
// n stages, spt stages per tile. At most ge CTAs take part, each a contiguous range of at least
// ceil(spt / (MAXC - 1)) stages, so at most MAXC CTAs touch any tile.
struct Split {
  int n, spt, ge;
  __host__ __device__ void init(int n_, int spt_, int G) {
    n = n_;
    spt = spt_;
    const int mn = (spt + MAXC - 2) / (MAXC - 1);
    ge = n / (mn > 0 ? mn : 1);
    ge = ge < 1 ? 1 : (ge > G ? G : ge);
  }
  // n * G stays below 2^32 for every supported shape (n <= 65 slots x 128 tiles x 64 blocks), so the
  // boundaries take 32-bit unsigned divisions.
  __host__ __device__ int lo(int c) const { return c < ge ? (int)((unsigned)n * (unsigned)c / (unsigned)ge) : n; }
  __host__ __device__ int hi(int c) const { return c < ge ? (int)((unsigned)n * (unsigned)(c + 1) / (unsigned)ge) : n; }
  __host__ __device__ int owner(int s) const {  // the CTA whose range holds stage s
    int c = (int)((unsigned)s * (unsigned)ge / (unsigned)(n > 0 ? n : 1));
    if (c >= ge) c = ge - 1;
    while (c + 1 < ge && lo(c + 1) <= s) ++c;
    while (c > 0 && lo(c) > s) --c;
    return c;
  }
};

// The four sequences of a launch (kinds 0..3) and the position of a CTA in them.
struct Work {
  Split sp[4];
  int nr;
  __device__ void init(const TcArgs& a, int nr_) {
    nr = nr_;
    const int G = gridDim.x;
    sp[0].init(a.P1 * a.KB1, a.KB1, G);
    sp[1].init(nr * a.P1 * a.KB1, a.KB1, G);
    sp[2].init(a.MT2 * a.KB2, a.KB2, G);
    sp[3].init(nr * a.MT2 * a.KB2, a.KB2, G);
  }
};

struct TcPlan {
  int nr;                 // routed slots
  int expert[MAXSLOT];    // slot -> routed expert
  float w[MAXSLOT][MAXB]; // routing weight of slot s for token t (0 when t did not choose it)
  int sel[MAXB][MAXK];
  float selw[MAXB][MAXK];
  float xscale[MAXB];
  Work wk;                // the launch's four stream-K splits (after the plan)
  unsigned long long* cnt13;  // this launch's counter set (see TcArgs::cnt)
  unsigned long long* cnt2;
  unsigned long long* sdone;
  int efl;                // epilogue: what the unit just closed leaves to finish (0, 1 = w1|w3 tile, 2 = w2 tile)
  unsigned tag;           // this launch's number + 1
  unsigned ar_epoch;
  volatile int ready;     // plan published (producer, helpers)
  volatile int abort;
};

// A unit: one CTA's contiguous run of K blocks inside one tile of one sequence (kinds 0..3 =
// shared w1|w3, routed w1|w3, shared w2, routed w2). Each CTA's units are listed once per launch in
// shared memory; every pipeline role walks that list, stage by stage, with register-only loops.
struct Unit {
  short kind, slot;  // slot: routed slot, or -1 for the shared expert
  short tile, j0;    // w1|w3: 64-row tile p; w2: output tile m; first K block
  short n, jc;       // K blocks; this CTA's contributor index within the tile
  int expert;        // routed expert (0 for the shared expert)
  int tile_id;       // tile index within the kind's sequence
};
constexpr int UMAX = 48;  // units per kind and CTA (the splits give at most about 20)

__device__ __forceinline__ int contrib_count(const Split& sp, int tile_id) {
  return sp.owner(tile_id * sp.spt + sp.spt - 1) - sp.owner(tile_id * sp.spt) + 1;
}

// ------------------------------------------------------------------ small device helpers
__device__ __forceinline__ unsigned long long ld_relaxed64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long atom_add_acq_rel(unsigned long long* p, unsigned long long v) {
  unsigned long long old;
  asm volatile("atom.add.acq_rel.gpu.global.u64 %0, [%1], %2;" : "=l"(old) : "l"(p), "l"(v) : "memory");
  return old;
}
__device__ __forceinline__ void red_add_release(unsigned long long* p, unsigned long long v) {
  asm volatile("red.add.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// L2 prefetch of a contiguous range (16-byte aligned start, size a multiple of 16 bytes).
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes & ~15u) : "memory");
}
__device__ __forceinline__ void st_relaxed64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_relaxed32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ float fscore_tc(float l, int func) {
  const double d = (double)l;
  const double s = func == DSMOE_SCORE_SIGMOID ? 1.0 / (1.0 + exp(-d)) : sqrt(d > 20.0 ? d : log1p(exp(d)));
  return __double2float_rn(s);
}
__device__ __forceinline__ unsigned score_key_tc(float f) {
  const unsigned u = f == 0.f ? 0u : __float_as_uint(f);
  return f != f ? 0u : u ^ ((unsigned)((int)u >> 31) | 0x80000000u);
}
__device__ __forceinline__ float silu_tc(float v) { return v / (1.0f + expf(-v)); }

// Offset of 16-byte chunk cc (0..7) of row r in a K-major SW128 tile with 128-byte rows.
__device__ __forceinline__ uint32_t sw128_off(int r, int cc) { return (uint32_t)(r * 128 + ((cc ^ (r & 7)) << 4)); }

// Named barrier whose participants all get the OR of their predicates: decisions taken after it are
// the same in every participating warp (so no warp leaves a barrier sequence the others are in).
__device__ __forceinline__ bool bar_any(int id, int n, bool p) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.or.pred q, %2, %3, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r) : "r"((uint32_t)p), "r"(id), "r"(n) : "memory");
  return r != 0;
}

// ------------------------------------------------------------------ tcgen05 / TMA wrappers
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void mma_f8(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void mma_mx(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t sfa, uint32_t sfb,
                                       uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb));
}
// Tensor-memory loads; the wait is inside the same statement, so no use of the registers can be
// scheduled before the data has arrived.
__device__ __forceinline__ void tm_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// Two 16-column accumulators (any two addresses) with one wait.
__device__ __forceinline__ void tm_ld16x2(uint32_t ta, uint32_t tb, float (&va)[16], float (&vb)[16]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%32];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%33];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(ta), "r"(tb)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    va[i] = __uint_as_float(r[i]);
    vb[i] = __uint_as_float(r[16 + i]);
  }
}
__device__ __forceinline__ void tm_st4(uint32_t taddr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tma_4d(void* dst, const CUtensorMap* tm, int c0, int c1, int c2, int c3, uint64_t* bar,
                                       uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

// ------------------------------------------------------------------ shared-memory carve-up
struct TcSmem {
  size_t efin, ring, xb, scr, bars, plan, emask, etab, fin, queue, units, misc, total;
};
__host__ __device__ inline TcSmem tc_smem(int H, int S, int E, int B) {
  TcSmem L;
  size_t o = 0;
  L.ring = o;
  o += (size_t)S * STAGE;
  L.xb = o;  // the w1|w3 B tile
  o += (size_t)(H / 128) * 2048;
  L.scr = o;  // the plan's scores and biased scores, [B][E] each
  o += ((size_t)2 * B * E * 4 + 15) & ~size_t(15);
  L.bars = o;
  o += (size_t)(3 * S + 2 * NACC8 + 5 * NISS + 1) * 8;
  o = (o + 15) & ~size_t(15);
  L.plan = o;
  o += (sizeof(TcPlan) + 15) & ~size_t(15);
  L.emask = o;
  o += (size_t)MAXE * 4;
  L.etab = o;
  o += 2 * 256 * 4;  // two units' FP8 scale tables: 4 floats per 128-K block, <= 64 blocks
  L.fin = o;
  o += 128 * 8 * 4;
  L.efin = o;  // the epilogue's finishing scratch: [64][8] + [8][64] floats, then [MAXSLOT] counts
  o += 2 * 64 * 8 * 4 + ((MAXSLOT * 4 + 15) & ~15);
  L.queue = o;
  o += (QCAP + 4) * 4;
  L.units = o;
  o += 4 * UMAX * sizeof(Unit) + 16;
  L.misc = o;
  o += 64;
  L.total = o + 1024;  // + alignment slack of the dynamic shared memory base
  return L;
}

// ------------------------------------------------------------------ router (warps 2..7)
// Quarter-rows of the router spread over the CTAs: H / 4 fp32 weights of a quarter-row in a warp's
// registers, the dot product with every token in fp64 (each product exact), stored as a tagged
// partial that every CTA's plan gathers.
__device__ __forceinline__ void warp_sum_d2(double& u, double& v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const double su = __shfl_xor_sync(0xffffffffu, u, o), sv = __shfl_xor_sync(0xffffffffu, v, o);
    u += su;
    v += sv;
  }
}
// Two quarter-rows per warp pass, interleaved: both rows' weights and the first token's values for
// both are loaded before any is used, and the two dot products share their latency chains. NI =
// float4 per lane of a quarter-row (H / 512, rounded up).
template <int NI>
__device__ __noinline__ void router_rows_t(const TcArgs& a, int w, int nw, int lane, int s0, int s1, double* qs) {
  const int n4 = a.H / 16;  // float4 per quarter-row
  for (int it0 = s0 + 2 * w; it0 < s1; it0 += 2 * nw) {
    const bool two = it0 + 1 < s1;
    float4 wv[2][NI];
    uint2 xv[2][NI];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int it = it0 + h;
      const float4* wrow = reinterpret_cast<const float4*>(a.wg + (long long)(it >> 2) * a.H + (it & 3) * (a.H / 4));
      const __nv_bfloat16* xr = a.x + (it & 3) * (a.H / 4);
#pragma unroll
      for (int i = 0; i < NI; ++i) {
        const int f = lane + 32 * i;
        if ((h == 0 || two) && f < n4) {
          const uint4 u = ld_stream16(wrow + f);
          wv[h][i] = make_float4(__uint_as_float(u.x), __uint_as_float(u.y), __uint_as_float(u.z), __uint_as_float(u.w));
          xv[h][i] = *reinterpret_cast<const uint2*>(xr + 4 * f);
        } else {
          wv[h][i] = make_float4(0.f, 0.f, 0.f, 0.f);
          xv[h][i] = make_uint2(0u, 0u);
        }
      }
    }
    for (int b = 0; b < a.B; ++b) {
      if (b > 0) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const __nv_bfloat16* xr = a.x + (long long)b * a.H + ((it0 + h) & 3) * (a.H / 4);
#pragma unroll
          for (int i = 0; i < NI; ++i) {
            const int f = lane + 32 * i;
            if ((h == 0 || two) && f < n4) xv[h][i] = *reinterpret_cast<const uint2*>(xr + 4 * f);
          }
        }
      }
      double acc[2][4];
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[h][c] = 0.0;
#pragma unroll
      for (int i = 0; i < NI; ++i)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint2 u = xv[h][i];
          acc[h][0] = fma((double)__uint_as_float(u.x << 16), (double)wv[h][i].x, acc[h][0]);
          acc[h][1] = fma((double)__uint_as_float(u.x & 0xFFFF0000u), (double)wv[h][i].y, acc[h][1]);
          acc[h][2] = fma((double)__uint_as_float(u.y << 16), (double)wv[h][i].z, acc[h][2]);
          acc[h][3] = fma((double)__uint_as_float(u.y & 0xFFFF0000u), (double)wv[h][i].w, acc[h][3]);
        }
      double v0 = (acc[0][0] + acc[0][1]) + (acc[0][2] + acc[0][3]);
      double v1 = (acc[1][0] + acc[1][1]) + (acc[1][2] + acc[1][3]);
      warp_sum_d2(v0, v1);
      if (lane == 0) {
        qs[(it0 - s0) * MAXB + b] = v0;
        if (two) qs[(it0 + 1 - s0) * MAXB + b] = v1;
      }
    }
  }
}
// This CTA's share of the router, rows [E c / G, E (c + 1) / G): fp32 weights times bf16 tokens,
// each product exact in fp64 and summed in fp64 per quarter-row (warps w = 0..nw-1, named barrier 4),
// the four quarters added in order, rounded to fp32 and scored; published as one tagged 8-byte word
// (launch tag, fp32 score) per (token, expert). qs: shared scratch of [4 rows][MAXB] doubles.
__device__ __noinline__ void router_rows(const TcArgs& a, TcPlan& pl, int w, int nw, int lane, double* qs) {
  const int G = gridDim.x;
  const int r0 = (int)((unsigned)a.E * (unsigned)blockIdx.x / (unsigned)G);
  const int r1 = (int)((unsigned)a.E * (unsigned)(blockIdx.x + 1) / (unsigned)G);
  if (a.H <= 5120)
    router_rows_t<10>(a, w, nw, lane, 4 * r0, 4 * r1, qs);
  else
    router_rows_t<16>(a, w, nw, lane, 4 * r0, 4 * r1, qs);
  named_bar_sync(4, 32 * nw);
  const unsigned long long tg = (unsigned long long)pl.tag << 32;
  for (int i = 32 * w + lane; i < (r1 - r0) * a.B; i += 32 * nw) {
    const int rr = i / a.B, b = i - rr * a.B;
    const double* q = qs + 4 * rr * MAXB + b;
    const float sc = fscore_tc(__double2float_rn(((q[0] + q[MAXB]) + q[2 * MAXB]) + q[3 * MAXB]), a.score_func);
    st_relaxed64(a.rl + (long long)b * a.E + r0 + rr, tg | __float_as_uint(sc));
  }
  named_bar_sync(4, 32 * nw);  // qs is read above; the warps reuse that memory afterwards
}

// ------------------------------------------------------------------ plan (warps 2-3, 64 threads)
// Scores of every (token, expert) from the tagged router partials (polled, bounded), top-k per token
// (ties -> lower index), weights / (sum + 1e-20) * route_scale, then the slots: the experts any token
// chose, in expert order, each with its per-token routing weight. sc / bi: [B][E] scratch.
// Top-k of token b (one warp): experts lane + 32 j, j < NJ, as order-preserving keys in registers,
// each packed with its j (lower j wins a tie) so that a lane's best is a depth-log2(NJ) max tree;
// then the warp's best key and, among lanes holding it, the lowest expert. Ties go to the lower
// expert index. Weights: score / (sum + 1e-20) * route_scale.
template <int NJ>
__device__ void topk_token(const TcArgs& a, TcPlan& pl, const float* sc, const float* bi, int b, int lane) {
  const float* v = bi + b * a.E;
  unsigned long long pk[NJ];
#pragma unroll
  for (int j = 0; j < NJ; ++j)
    pk[j] = lane + 32 * j < a.E ? ((unsigned long long)score_key_tc(v[lane + 32 * j]) << 32) | (unsigned)(NJ - 1 - j) : 0ull;
  unsigned mine = 0u;
  for (int r = 0; r < a.topk; ++r) {
    unsigned long long t[NJ];
#pragma unroll
    for (int j = 0; j < NJ; ++j) t[j] = pk[j];
#pragma unroll
    for (int w = NJ / 2; w >= 1; w /= 2)
#pragma unroll
      for (int j = 0; j < w; ++j) t[j] = t[j] > t[j + w] ? t[j] : t[j + w];
    const unsigned bk = (unsigned)(t[0] >> 32);
    const int bj = NJ - 1 - (int)(t[0] & 0xFFFFu);
    const unsigned m = __reduce_max_sync(0xffffffffu, bk);
    unsigned bi_ = __reduce_min_sync(0xffffffffu, bk == m ? (unsigned)(lane + 32 * bj) : 0xFFFFFFFFu);
    if (bi_ >= (unsigned)a.E) bi_ = 0u;
    if (lane == r) mine = bi_;
    if (lane == (int)(bi_ & 31u)) {
#pragma unroll
      for (int j = 0; j < NJ; ++j)
        if (j == (int)(bi_ >> 5)) pk[j] = 0ull;
    }
  }
  const float wv = lane < a.topk ? sc[b * a.E + mine] : 0.f;
  float tot = 0.f;
  for (int r = 0; r < a.topk; ++r) tot += __shfl_sync(0xffffffffu, wv, r);
  if (lane < a.topk) {
    const float w = wv / (tot + 1e-20f) * a.route_scale;
    pl.sel[b][lane] = (int)mine;
    pl.selw[b][lane] = w;
    if (blockIdx.x == 0) {
      if (a.idx) a.idx[b * a.topk + lane] = mine;
      if (a.wt) a.wt[b * a.topk + lane] = w;
    }
  }
}

constexpr int PT = 64, BAR_PLAN = 3;  // plan threads (warps 2 and 3) and their named barrier
__device__ __noinline__ bool make_plan(const TcArgs& a, TcPlan& pl, float* sc, float* bi, unsigned* emask, int t7) {
  const int w7 = t7 >> 5, lane = t7 & 31;
  const int n = a.B * a.E;
  const unsigned tag = pl.tag;
  const uint64_t t0 = globaltimer_ns();
  // Eight (token, expert) scores per thread and pass, their tagged words and biases all loaded before
  // any is checked: one memory round trip per pass once every CTA has published its rows.
  constexpr int NB = 8;
  for (int i0 = t7; i0 < n; i0 += NB * PT) {
    unsigned long long w[NB];
    float bs[NB];
    unsigned need = 0u;
#pragma unroll
    for (int u = 0; u < NB; ++u) {
      const int i = i0 + u * PT;
      if (i < n) {
        need |= 1u << u;
        const int b = i / a.E, e = i - b * a.E;
        const bool vl = a.bias_vl != nullptr && a.image_mask != nullptr && a.image_mask[b] != 0;
        bs[u] = (vl ? a.bias_vl : a.bias)[e];
      }
    }
    while (need != 0u) {
#pragma unroll
      for (int u = 0; u < NB; ++u)
        if ((need >> u) & 1u) w[u] = ld_relaxed64(a.rl + i0 + u * PT);
#pragma unroll
      for (int u = 0; u < NB; ++u)
        if (((need >> u) & 1u) && (unsigned)(w[u] >> 32) == tag) {
          const float sv = __uint_as_float((unsigned)w[u]);
          sc[i0 + u * PT] = sv;
          bi[i0 + u * PT] = sv + bs[u];
          need &= ~(1u << u);
        }
      if (need != 0u && (ld_relaxed32(a.status) != 0u || globaltimer_ns() - t0 > kWait)) {
        atomicOr(a.status, ST_PLAN);
        pl.abort = 1;
        break;
      }
    }
    if (need != 0u) break;
  }
  if (bar_any(BAR_PLAN, PT, pl.abort != 0)) return false;
  if (blockIdx.x == 0 && a.scores)
    for (int i = t7; i < n; i += PT) a.scores[i] = sc[i];
  // top-k of token b by warp b % 2: keys of the lane's experts (lane + 32 j) in registers
  for (int b = w7; b < a.B; b += PT / 32) {
    if (a.E <= 128)
      topk_token<4>(a, pl, sc, bi, b, lane);
    else if (a.E <= 256)
      topk_token<8>(a, pl, sc, bi, b, lane);
    else if (a.E <= 512)
      topk_token<16>(a, pl, sc, bi, b, lane);
    else
      topk_token<32>(a, pl, sc, bi, b, lane);
  }
  named_bar_sync(BAR_PLAN, PT);
  if (a.B == 1) {
    // one token: its k distinct picks are the slots, in expert order
    if (w7 == 0 && lane < a.topk) {
      const int e = pl.sel[0][lane];
      int rk = 0;
      for (int r = 0; r < a.topk; ++r) rk += pl.sel[0][r] < e ? 1 : 0;
      pl.expert[rk] = e;
      pl.w[rk][0] = pl.selw[0][lane];
      for (int t = 1; t < MAXB; ++t) pl.w[rk][t] = 0.f;
    }
    if (t7 == 0) pl.nr = a.topk;
  } else {
    for (int e = t7; e < a.E; e += PT) emask[e] = 0u;
    named_bar_sync(BAR_PLAN, PT);
    for (int i = t7; i < a.B * a.topk; i += PT) atomicOr(&emask[pl.sel[i / a.topk][i % a.topk]], 1u << (i / a.topk));
    named_bar_sync(BAR_PLAN, PT);
    if (w7 == 0) {  // compaction in expert order, 32 experts per step
      int base = 0;
      for (int e0 = 0; e0 < a.E; e0 += 32) {
        const int e = e0 + lane;
        const unsigned m = e < a.E ? emask[e] : 0u;
        const unsigned bal = __ballot_sync(0xffffffffu, m != 0u);
        if (m != 0u) {
          const int s = base + __popc(bal & ((1u << lane) - 1u));
          pl.expert[s] = e;
          for (int t = 0; t < MAXB; ++t) {
            float w = 0.f;
            if (t < a.B && ((m >> t) & 1u))
              for (int r = 0; r < a.topk; ++r)
                if (pl.sel[t][r] == e) w = pl.selw[t][r];
            pl.w[s][t] = w;
          }
        }
        base += __popc(bal);
      }
      if (lane == 0) pl.nr = base;
    }
  }
  named_bar_sync(BAR_PLAN, PT);
  return true;
}

// Token rows -> per-token power-of-two pre-scale (amax 2^-p in [128, 256)) -> the MMA's B tile of
// the w1|w3 phase: [H / 128 blocks][16 rows][128 B], K-major SW128; row t < 8 holds the e4m3 "hi"
// part of token t, row 8 + t its "lo" part (x 2^-p ~ hi + lo / 16); rows of tokens >= B are zero.
// 224 threads (warps 1-7); thread t7 owns the 16-element chunk columns c = t7 + 224 r of every token.
// With up to XBT tokens and XC columns a thread (H <= 7168) the chunks are loaded once, all before
// their first use, and stay in registers; otherwise the conversion loads them again.
constexpr int XT = 224, XC = 2, XBT = 4;
__device__ __forceinline__ float amax16(const uint4& u0, const uint4& u1) {
  const uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
  float m = 0.f;
#pragma unroll
  for (int h = 0; h < 8; ++h)
    m = fmaxf(m, fmaxf(fabsf(__uint_as_float(w[h] << 16)), fabsf(__uint_as_float(w[h] & 0xFFFF0000u))));
  return m;
}
__device__ __forceinline__ void put_xb(uint8_t* xb, int b, int c, float inv, const uint4& u0, const uint4& u1) {
  uint32_t hw[4] = {0u, 0u, 0u, 0u}, lw[4] = {0u, 0u, 0u, 0u};
  const uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
  for (int h = 0; h < 8; ++h) {
    uint32_t h2, l2;
    split2_e4m3(__uint_as_float(w[h] << 16) * inv, __uint_as_float(w[h] & 0xFFFF0000u) * inv, h2, l2);
    hw[h >> 1] |= h2 << (16 * (h & 1));
    lw[h >> 1] |= l2 << (16 * (h & 1));
  }
  uint8_t* blk = xb + (size_t)(c >> 3) * 2048;
  *reinterpret_cast<uint4*>(blk + sw128_off(b, c & 7)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
  *reinterpret_cast<uint4*>(blk + sw128_off(8 + b, c & 7)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
}
__device__ __noinline__ void build_xb(const TcArgs& a, uint8_t* xb, TcPlan& pl, float* red, int t7) {
  const int w7 = t7 >> 5, lane = t7 & 31;
  const int nc = a.H / 16;
  const bool keep = nc <= XT * XC && a.B <= XBT;
  uint4 v[XBT][XC][2];
  if (keep) {
#pragma unroll
    for (int b = 0; b < XBT; ++b)
#pragma unroll
      for (int r = 0; r < XC; ++r) {
        const int c = t7 + XT * r;
        if (b < a.B && c < nc) {
          const uint4* src = reinterpret_cast<const uint4*>(a.x + (long long)b * a.H + 16 * c);
          v[b][r][0] = src[0];
          v[b][r][1] = src[1];
        }
      }
  }
  // the whole tile to zero while the loads are in flight (the rows of absent tokens stay zero)
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);
  for (int o = t7; o < a.KB1 * 128; o += XT) reinterpret_cast<uint4*>(xb)[o] = z;
  if (keep) {
#pragma unroll
    for (int b = 0; b < XBT; ++b) {
      if (b >= a.B) break;
      float m = 0.f;
#pragma unroll
      for (int r = 0; r < XC; ++r)
        if (t7 + XT * r < nc) m = fmaxf(m, amax16(v[b][r][0], v[b][r][1]));
      m = warp_max(m);
      if (lane == 0) red[b * 8 + w7] = m;
    }
  } else {
    for (int b = 0; b < a.B; ++b) {
      const uint4* src = reinterpret_cast<const uint4*>(a.x + (long long)b * a.H);
      float m = 0.f;
      for (int c = t7; c < nc; c += XT) m = fmaxf(m, amax16(src[2 * c], src[2 * c + 1]));
      m = warp_max(m);
      if (lane == 0) red[b * 8 + w7] = m;
    }
  }
  named_bar_sync(1, XT);
  if (t7 < a.B) {
    float m = 0.f;
    for (int w = 0; w < 7; ++w) m = fmaxf(m, red[t7 * 8 + w]);
    int p = 0;
    if (m > 0.f && m <= 3.0e38f) {
      int e2;
      frexpf(m, &e2);
      p = e2 - 8;
    }
    pl.xscale[t7] = ldexpf(1.0f, p);
  }
  named_bar_sync(1, XT);
  if (keep) {
#pragma unroll
    for (int b = 0; b < XBT; ++b) {
      if (b >= a.B) break;
      const float inv = 1.0f / pl.xscale[b];
#pragma unroll
      for (int r = 0; r < XC; ++r)
        if (t7 + XT * r < nc) put_xb(xb, b, t7 + XT * r, inv, v[b][r][0], v[b][r][1]);
    }
  } else {
    for (int b = 0; b < a.B; ++b) {
      const uint4* src = reinterpret_cast<const uint4*>(a.x + (long long)b * a.H);
      const float inv = 1.0f / pl.xscale[b];
      for (int c = t7; c < nc; c += XT) put_xb(xb, b, c, inv, src[2 * c], src[2 * c + 1]);
    }
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> the tensor core's reads
  named_bar_sync(1, XT);
}

// ------------------------------------------------------------------ pipeline state in shared memory
struct Pipe {
  uint8_t* ring;
  uint8_t* xb;
  uint64_t* full;   // [S] stage bytes landed (A, FP4 scales, and the B tile of a w2 stage)
  uint64_t* empty;  // [S] stage consumed by the MMAs
  uint64_t* sfr;    // [S] FP4 scale factors of the stage in tensor memory (4 epilogue warps); one phase
                    // per FP4 stage of the slot only
  uint64_t* accf;   // [NACC8] FP8 block accumulator complete
  uint64_t* accr;   // [NACC8] FP8 block accumulator read (4 epilogue warps)
  uint64_t* a4f;    // [2 parities][NISS] FP4 unit accumulator of an issuer complete
  uint64_t* a4r;    // [2 parities][NISS] FP4 unit accumulator of an issuer read (4 epilogue warps)
  uint64_t* mdone;  // [NISS] every MMA of an issuer complete
  uint64_t* rdy;    // the plan and the routed units are published (one arrival)
  int* queue;       // [QCAP] finisher jobs
  volatile int* qtail;
  volatile int* edone;   // the epilogue has queued its last job
  volatile int* issued;  // stages armed by the producer
  const Unit* units;     // [4][UMAX]
  const int* ucnt;       // [4]
  uint32_t tm;
  int S;
};

__device__ __forceinline__ bool pwait(const TcArgs& a, TcPlan& pl, uint64_t* bar, uint32_t par) {
  if (pl.abort) return false;
  if (!mbar_wait(bar, par, kWait)) {
    atomicOr(a.status, ST_MBAR);
    pl.abort = 1;
    return false;
  }
  return true;
}

// FP8 scale segment of K step k of block j: the 128-K block of the full expert it falls in. A
// segment of a w2 stage may continue into the next stage when the slice starts inside a block.
__device__ __forceinline__ int seg_key(int row0, int kind, int j, int k) {
  return kind < 2 ? j : (row0 + 128 * j + 32 * k) >> 7;
}
__device__ __forceinline__ int seg_next(int row0, int kind, int j) {
  return kind < 2 ? j + 1 : (row0 + 128 * (j + 1)) >> 7;
}
__device__ __forceinline__ int ksteps(int I_loc, int kind, int j) { return kind < 2 ? 4 : min(4, (I_loc - 128 * j) / 32); }
__device__ __forceinline__ bool last_of(const Unit& U, int j) { return j == U.j0 + U.n - 1; }

// Position in a CTA's stream: (kind, unit, K block) and the ring stage g.
struct Cur {
  int k, u, j, g;
  __device__ void start(const Pipe& P, int kmin, int g0) {
    k = kmin;
    u = 0;
    j = 0;
    g = g0;
    settle(P);
  }
  __device__ void settle(const Pipe& P) {  // to the first block of the current or a later unit
    while (k < 4 && u >= P.ucnt[k]) {
      ++k;
      u = 0;
    }
    if (k < 4) j = P.units[k * UMAX + u].j0;
  }
  __device__ bool valid() const { return k < 4; }
  __device__ void next(const Pipe& P) {
    const Unit& U = P.units[k * UMAX + u];
    ++g;
    if (++j >= U.j0 + U.n) {
      ++u;
      settle(P);
    }
  }
};

// Polls of shared or global words spin without sleeping: a sleeping thread wakes up late (measured
// here at over a microsecond), and every such wait sits on the layer's critical path.
__device__ __forceinline__ void backoff() {}

// Waits (bounded) until the plan and the routed units are published: the plan thread arrives on the
// `rdy` barrier (release), the waiters' try_wait acquires.
__device__ void wait_ready(const TcArgs& a, TcPlan& pl, uint64_t* rdy) {
  if (!mbar_wait(rdy, 0, kWait)) {
    atomicOr(a.status, ST_PLAN);
    pl.abort = 1;
  }
}

// ---- warp 0, lane 0: TMA producer. One 128 x 128 tensor box per stage (plus an FP4 block's scales).
__device__ __noinline__ void role_producer(const TcArgs& a, TcPlan& pl, const Pipe& Pin) {
  const Pipe P = Pin;
  const uint64_t pol = l2_evict_first();
  // the four tensor maps into the TMA unit's descriptor cache now, not at their first copies
  asm volatile("prefetch.tensormap [%0];" ::"l"(&a.tm_s13) : "memory");
  asm volatile("prefetch.tensormap [%0];" ::"l"(&a.tm_r13) : "memory");
  asm volatile("prefetch.tensormap [%0];" ::"l"(&a.tm_s2) : "memory");
  asm volatile("prefetch.tensormap [%0];" ::"l"(&a.tm_r2) : "memory");
  int slot = 0, ph = 0, g = 0;
  for (int k = 0; k < 4 && !pl.abort; ++k) {
    if (k == 1) {  // routed work needs the plan
      wait_ready(a, pl, P.rdy);
      if (pl.abort) break;
    }
    const bool w13 = k < 2, routed = k & 1;
    const bool f4 = routed && a.r_fmt == DSMOE_FMT_FP4;
    const CUtensorMap* tm = w13 ? (routed ? &a.tm_r13 : &a.tm_s13) : (routed ? &a.tm_r2 : &a.tm_s2);
    const int per = w13 ? a.KB1 : a.KB2;
    const uint32_t bytes = (f4 ? 8192u + 512u : (uint32_t)SA) + (w13 ? 0u : (uint32_t)SB);
    const int nu = P.ucnt[k];
    for (int u = 0; u < nu && !pl.abort; ++u) {
      const Unit U = P.units[k * UMAX + u];
      const uint8_t* eb = w13 ? a.r13 + (long long)U.expert * a.r_eb13 : a.r2 + (long long)U.expert * a.r_eb2;
      for (int j = U.j0; j < U.j0 + U.n; ++j) {
        // At most `depth` stages in flight: the weight bytes HBM needs to run at full rate (about 64 KB a
        // SM), and no more, since every extra byte in flight is queueing delay for the kernel's other
        // memory traffic (router, partials, exchange).
        const int depth = f4 ? P.S : min(P.S, kDepth8);
        if (g >= depth) {
          const int q = g - depth;
          if (!pwait(a, pl, &P.empty[q % P.S], (q / P.S) & 1)) break;
        }
        // the two MMA issuers may release stages out of order: the slot itself must be free too
        if (g >= P.S && !pwait(a, pl, &P.empty[slot], ph ^ 1)) break;
        uint8_t* A = P.ring + (size_t)slot * STAGE;
        const int blk = U.tile * per + j;
        mbar_expect_tx(&P.full[slot], bytes);
        tma_4d(A, tm, 0, 0, blk, U.expert, &P.full[slot], pol);
        if (f4) bulk_g2s_hint(A + SA + SB, eb + (long long)blk * (8192 + 512) + 8192, 512, &P.full[slot], pol);
        ++g;
        *P.issued = g;
        if (++slot == P.S) {
          slot = 0;
          ph ^= 1;
        }
      }
    }
  }
  // every copy issued lands before the CTA may exit (the MMAs consumed all of them unless aborted)
  for (int q = max(0, g - P.S); q < g; ++q) mbar_wait(&P.full[q % P.S], (q / P.S) & 1, kWait);
}

// ---- warp 2, lane 0: the B tile (h of the slot) of every w2 stage, once the slot is finished
__device__ __noinline__ void role_hcopy(const TcArgs& a, TcPlan& pl, const Pipe& Pin, int SH) {
  const Pipe P = Pin;
  int g = 0;
  for (int k = 0; k < 2; ++k)
    for (int u = 0; u < P.ucnt[k]; ++u) g += P.units[k * UMAX + u].n;
  int slot = g % P.S;
  int ready_slot = -2;
  for (int k = 2; k < 4 && !pl.abort; ++k) {
    for (int u = 0; u < P.ucnt[k] && !pl.abort; ++u) {
      const Unit U = P.units[k * UMAX + u];
      const int si = U.slot < 0 ? SH : U.slot;
      for (int j = U.j0; j < U.j0 + U.n && !pl.abort; ++j) {
        const uint64_t t0 = globaltimer_ns();
        while (*P.issued <= g && !pl.abort) {  // the producer has armed this stage's barrier
          backoff();
          if (globaltimer_ns() - t0 > kWait) {
            atomicOr(a.status, ST_MBAR);
            pl.abort = 1;
          }
        }
        if (si != ready_slot) {
          while (ld_relaxed64(pl.sdone + si) < (unsigned long long)a.P1 && !pl.abort) {
            backoff();
            if (ld_relaxed32(a.status) != 0u || globaltimer_ns() - t0 > kWait) {
              atomicOr(a.status, ST_CNT);
              pl.abort = 1;
            }
          }
          if (pl.abort) break;
          fence_acq_rel_gpu();
          asm volatile("fence.proxy.async.global;" ::: "memory");
          ready_slot = si;
        }
        bulk_g2s(P.ring + (size_t)slot * STAGE + SA, a.hb + ((long long)si * a.KB2 + j) * 2048, SB, &P.full[slot]);
        ++g;
        if (++slot == P.S) slot = 0;
      }
    }
  }
}

// Instruction descriptors: FP8 x FP8 (kind::f8f6f4) and e2m1 x e4m3 with e8m0 block scales
// (kind::mxf8f6f4), both M = 128, N = 16, fp32 accumulate.
constexpr uint32_t kIdesc8 = (1u << 4) | ((16u >> 3) << 17) | ((128u >> 4) << 24);
constexpr uint32_t kIdescX = (5u << 7) | ((16u >> 3) << 17) | (1u << 23) | ((128u >> 4) << 24);

// The four 32-K MMAs of one stage, issued back to back. A 32-byte step along K is +2 in the start
// address field of a 128-byte-swizzled descriptor (stage bases are 1 KB aligned, so the field
// never carries); every operand is known before the first MMA goes out, which keeps the issuing
// thread's serial latency out of the tensor core's way.
__device__ __forceinline__ void mma4_f8(uint32_t d, uint64_t da, uint64_t db, uint32_t acc0) {
  mma_f8(d, da, db, kIdesc8, acc0);
  mma_f8(d, da + 2, db + 2, kIdesc8, 1u);
  mma_f8(d, da + 4, db + 4, kIdesc8, 1u);
  mma_f8(d, da + 6, db + 6, kIdesc8, 1u);
}
__device__ __forceinline__ void mma4_mx(uint32_t d, uint64_t da, uint64_t db, uint32_t sfa, uint32_t sfb,
                                        uint32_t acc0) {
  mma_mx(d, da, db, kIdescX, sfa, sfb, acc0);
  mma_mx(d, da + 2, db + 2, kIdescX | (1u << 29) | (1u << 4), sfa | (1u << 30), sfb | (1u << 30), 1u);
  mma_mx(d, da + 4, db + 4, kIdescX | (2u << 29) | (2u << 4), sfa | (2u << 30), sfb | (2u << 30), 1u);
  mma_mx(d, da + 6, db + 6, kIdescX | (3u << 29) | (3u << 4), sfa | (3u << 30), sfb | (3u << 30), 1u);
}

// ---- lane 0 of warp 1 (issuer 0) and, at N = 1, of warp 3 (issuer 1): MMA issuers. One issuing
// thread is bound by its own serial latency (about one 4-MMA stage per 0.25 us), so at N = 1 two
// threads issue alternate stages of the routed work: stage i of the stream after the shared w1|w3
// phase goes to issuer i % 2 (issuer 0 keeps the shared w1|w3 stages, and every w2 stage of a slice
// that starts inside a 128-row block, whose scale segments run across stages). The two never share
// an accumulator: FP8 segments are distinct per stage, FP4 units accumulate per issuer (the epilogue
// adds the two). At N > 1 warp 3 runs the finisher and issuer 0 takes every stage.
__device__ __noinline__ void role_mma(const TcArgs& a, TcPlan& pl, const Pipe& Pin, int iss) {
  const Pipe P = Pin;
  int slot = 0, ph = 0, nseg = 0, n4 = 0, cur_a = 0, cur_g = -1, gi = 0;
  int u4[2] = {0, 0};  // FP4 units of each accumulator parity this issuer has taken part in
  uint32_t c4 = 0u;    // FP4 uses per ring slot, mod 2 (bit s): the phases of its scale-factor barrier
  bool open = false, ok = true;
  const uint32_t ring = smem_u32(P.ring), xb = smem_u32(P.xb);
  const bool w2_aligned = (a.row0 & 127) == 0;  // every w2 stage is then one FP8 scale segment
  for (int k = 0; k < 4 && ok; ++k) {
    if (k == 1) {  // the routed units exist once the plan is published
      wait_ready(a, pl, P.rdy);
      if (pl.abort) break;
    }
    const bool f4 = (k & 1) && a.r_fmt == DSMOE_FMT_FP4;
    const bool dual = a.ar_world <= 1 && k >= 1 && (k < 2 || f4 || w2_aligned);
    const int nu = P.ucnt[k];
    for (int u = 0; u < nu && ok; ++u) {
      const Unit U = P.units[k * UMAX + u];
      // FP4: this issuer's stages of the unit are those of stream parity iss (all of them single-issue)
      const int jf = (!dual || (gi & 1) == iss) ? U.j0 : U.j0 + 1;  // this issuer's first and last block
      const int jl = U.j0 + U.n - 1 - ((dual && ((gi + U.n - 1) & 1) != iss) ? 1 : 0);
      const int par = n4 & 1;
      const uint32_t d4 = P.tm + TM_ACC4 + 16 * (2 * par + iss);
      if (f4 && jf <= jl) {  // the accumulator's previous unit has been read by the epilogue
        if (u4[par] >= 1 && !pwait(a, pl, &P.a4r[2 * par + iss], (u4[par] - 1) & 1)) {
          ok = false;
          break;
        }
        fence_after();
      }
      for (int j = U.j0; j < U.j0 + U.n; ++j) {
        const bool mine = k == 0 ? iss == 0 : (dual ? (gi & 1) == iss : iss == 0);
        if (mine) {
          if (!pwait(a, pl, &P.full[slot], ph)) {
            ok = false;
            break;
          }
          if (f4 && !pwait(a, pl, &P.sfr[slot], (c4 >> slot) & 1u)) {
            ok = false;
            break;
          }
          fence_after();
          const uint32_t aA = ring + slot * STAGE;
          const uint32_t bB = k < 2 ? xb + j * 2048 : aA + SA;
          const uint64_t da = desc_sw128(aA), db = desc_sw128(bB);
          const int nk = ksteps(a.I_loc, k, j);
          if (f4) {
            const uint32_t sfa = P.tm + TM_SFA + 4 * slot, sfb = P.tm + TM_SFB;
            if (nk == 4) {
              mma4_mx(d4, da, db, sfa, sfb, j == jf ? 0u : 1u);
            } else {
              for (int q = 0; q < nk; ++q)
                mma_mx(d4, da + 2 * q, db + 2 * q, kIdescX | ((uint32_t)q << 29) | ((uint32_t)q << 4),
                       sfa | ((uint32_t)q << 30), sfb | ((uint32_t)q << 30), (j == jf && q == 0) ? 0u : 1u);
            }
            commit(&P.empty[slot]);
            if (j == jl) commit(&P.a4f[2 * par + iss]);
          } else if (k < 2 || w2_aligned) {  // the stage is exactly one scale segment
            cur_a = nseg & (NACC8 - 1);
            if (nseg >= NACC8) {
              if (!pwait(a, pl, &P.accr[cur_a], ((nseg / NACC8) - 1) & 1)) {
                ok = false;
                break;
              }
              fence_after();
            }
            if (nk == 4) {
              mma4_f8(P.tm + 16 * cur_a, da, db, 0u);
            } else {
              for (int q = 0; q < nk; ++q) mma_f8(P.tm + 16 * cur_a, da + 2 * q, db + 2 * q, kIdesc8, q == 0 ? 0u : 1u);
            }
            commit(&P.empty[slot]);
            commit(&P.accf[cur_a]);
          } else {  // w2 of a slice that starts inside a 128-row block (issuer 0 only): segments change mid-stage
            for (int q = 0; q < nk; ++q) {
              const int gk = seg_key(a.row0, k, j, q);
              bool fresh = false;
              if (!open || gk != cur_g) {
                if (open) commit(&P.accf[cur_a]);
                cur_a = nseg & (NACC8 - 1);
                if (nseg >= NACC8) {
                  if (!pwait(a, pl, &P.accr[cur_a], ((nseg / NACC8) - 1) & 1)) {
                    ok = false;
                    break;
                  }
                  fence_after();
                }
                ++nseg;
                cur_g = gk;
                open = true;
                fresh = true;
              }
              mma_f8(P.tm + 16 * cur_a, da + 2 * q, db + 2 * q, kIdesc8, fresh ? 0u : 1u);
            }
            if (!ok) break;
            commit(&P.empty[slot]);
            if (last_of(U, j) || seg_next(a.row0, k, j) != cur_g) {  // the segment does not continue into the next stage
              commit(&P.accf[cur_a]);
              open = false;
            }
          }
        }
        // both issuers follow the whole stream: ring position, FP8 segment count, FP4 slot phases
        if (f4) c4 ^= 1u << slot;
        else if (k < 2 || w2_aligned) ++nseg;
        if (k >= 1) ++gi;
        if (++slot == P.S) {
          slot = 0;
          ph ^= 1;
        }
      }
      if (f4) {
        if (jf <= jl) ++u4[par];
        ++n4;
      }
    }
  }
  commit(&P.mdone[iss]);  // completes once every MMA this thread issued has
  mbar_wait(&P.mdone[iss], 0, kWait);
}

// ---- finishing by the last contributor's epilogue (warps 4-7, 128 threads, named barrier 2)
// w1|w3 tile p of slot index si: the tile's partials summed in contributor order (this CTA's own from
// registers, the others' rows loaded together), h = SiLU(min(g, 10)) * clamp(u, +-10) * kHScale for
// its 64 intermediate rows (gate row r in thread r, up row in thread 64 + r), as e4m3 hi / lo bytes
// into the slot's w2 B tile; then the slot's count of finished tiles.
__device__ __noinline__ void epi_finish_w13(const TcArgs& a, TcPlan& pl, int kind, int si, int p, int tile_id, int jc,
                                            const float (&own)[MAXB], int m, float* ef) {
  const int nc = contrib_count(pl.wk.sp[kind], tile_id);
  const float* base = a.p13 + ((long long)si * a.P1 + p) * MAXC * 1024 + m * 8;
  uint4 v[MAXC][2];
#pragma unroll
  for (int j = 0; j < MAXC; ++j)
    if (j < nc && j != jc) {
      v[j][0] = ld_cg16(base + j * 1024);
      if (a.B > 4) v[j][1] = ld_cg16(base + j * 1024 + 4);
    }
  float s[MAXB];
#pragma unroll
  for (int t = 0; t < MAXB; ++t) s[t] = 0.f;
#pragma unroll
  for (int j = 0; j < MAXC; ++j)
    if (j < nc) {
      if (j == jc) {
#pragma unroll
        for (int t = 0; t < MAXB; ++t) s[t] += own[t];
      } else {
        s[0] += __uint_as_float(v[j][0].x);
        s[1] += __uint_as_float(v[j][0].y);
        s[2] += __uint_as_float(v[j][0].z);
        s[3] += __uint_as_float(v[j][0].w);
        if (a.B > 4) {
          s[4] += __uint_as_float(v[j][1].x);
          s[5] += __uint_as_float(v[j][1].y);
          s[6] += __uint_as_float(v[j][1].z);
          s[7] += __uint_as_float(v[j][1].w);
        }
      }
    }
  if (m >= 64) {
#pragma unroll
    for (int t = 0; t < MAXB; ++t) ef[(m - 64) * 8 + t] = s[t];
  }
  named_bar_sync(2, 128);
  float* hs = ef + 64 * 8;  // [token][row]
  if (m < 64) {
#pragma unroll
    for (int t = 0; t < MAXB; ++t) {
      const float gv = fminf(s[t], 10.0f);
      const float uv = fminf(fmaxf(ef[m * 8 + t], -10.0f), 10.0f);
      hs[t * 64 + m] = t < a.B ? silu_tc(gv) * uv * kHScale : 0.f;
    }
  }
  named_bar_sync(2, 128);
  // 16 B pieces: (B-tile row n = hi / lo of token n % 8, chunk of 16 K) -> SW128 position
  uint8_t* blk = a.hb + ((long long)si * a.KB2 + (p >> 1)) * 2048;
  const bool last_half = p == a.P1 - 1 && (p & 1) == 0;  // the block's second half lies past the slice: zero it
  if (m < 64 || last_half) {
    const int n = (m & 63) >> 2, c4 = m & 3;
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    if (m < 64) {
      const int t = n & 7;
      const bool lo = n >= 8;
      const float* hv = hs + t * 64 + 16 * c4;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        uint32_t h2, l2;
        split2_e4m3(hv[2 * q], hv[2 * q + 1], h2, l2);
        w[q >> 1] |= (lo ? l2 : h2) << (16 * (q & 1));
      }
    }
    const int cc = (m < 64 ? (p & 1) * 4 : 4) + c4;
    *reinterpret_cast<uint4*>(blk + sw128_off(n, cc)) = make_uint4(w[0], w[1], w[2], w[3]);
    asm volatile("fence.proxy.async.global;" ::: "memory");  // the B tile is read by bulk copies
  }
  named_bar_sync(2, 128);
  if (m == 0) red_add_release(pl.sdone + si, 1ull);  // release: every thread's B-tile bytes (ordered by the barrier)
}

// Output tile mt at N = 1: y rows [128 mt, 128 mt + 128) = the sum over the routed slots (in order)
// and the shared expert of their partials in contributor order; row m in thread m, CAP partial rows
// loaded together per pass (one pass for the usual 7 slots x 2 contributors).
template <int CAP, bool WIDE>
__device__ __forceinline__ void epi_sum_w2(const TcArgs& a, const float* base, const int* ecnt, int nl, int nr, int SH,
                                           float (&s)[MAXB]) {
  int li = 0, j = 0;
  while (li < nl) {
    uint4 v[CAP][WIDE ? 2 : 1];
    bool on[CAP];
#pragma unroll
    for (int q = 0; q < CAP; ++q) {
      while (li < nl && j >= ecnt[li]) {
        ++li;
        j = 0;
      }
      on[q] = li < nl;
      if (on[q]) {
        const float* src = base + ((long long)(li < nr ? li : SH) * MAXC + j) * 1024;
        v[q][0] = ld_cg16(src);
        if (WIDE) v[q][WIDE ? 1 : 0] = ld_cg16(src + 4);
        ++j;
      }
    }
#pragma unroll
    for (int q = 0; q < CAP; ++q)
      if (on[q]) {
        s[0] += __uint_as_float(v[q][0].x);
        s[1] += __uint_as_float(v[q][0].y);
        s[2] += __uint_as_float(v[q][0].z);
        s[3] += __uint_as_float(v[q][0].w);
        if (WIDE) {
          s[4] += __uint_as_float(v[q][WIDE ? 1 : 0].x);
          s[5] += __uint_as_float(v[q][WIDE ? 1 : 0].y);
          s[6] += __uint_as_float(v[q][WIDE ? 1 : 0].z);
          s[7] += __uint_as_float(v[q][WIDE ? 1 : 0].w);
        }
      }
  }
}
__device__ __noinline__ void epi_finish_w2(const TcArgs& a, TcPlan& pl, int mt, int SH, int m, int* ecnt) {
  const int nr = pl.nr, nl = nr + 1;
  for (int i = m; i < nl; i += 128) ecnt[i] = contrib_count(pl.wk.sp[i < nr ? 3 : 2], i < nr ? i * a.MT2 + mt : mt);
  named_bar_sync(2, 128);
  const float* base = a.p2 + (long long)mt * a.slot_cap * MAXC * 1024 + m * 8;
  float s[MAXB];
#pragma unroll
  for (int t = 0; t < MAXB; ++t) s[t] = 0.f;
  if (a.B > 4)
    epi_sum_w2<8, true>(a, base, ecnt, nl, nr, SH, s);
  else
    epi_sum_w2<16, false>(a, base, ecnt, nl, nr, SH, s);
#pragma unroll
  for (int t = 0; t < MAXB; ++t) {
    if (t >= a.B) break;
    const long long o = (long long)t * a.H + 128 * mt + m;
    if (a.y_f32)
      reinterpret_cast<float*>(a.y)[o] = s[t];
    else
      reinterpret_cast<__nv_bfloat16*>(a.y)[o] = __float2bfloat16_rn(s[t]);
  }
}

// ---- warps 4-7: epilogue. Thread = accumulator row m = 32 q + lane (TMEM lane quadrant q).
__device__ __noinline__ void role_epilogue(const TcArgs& a, TcPlan& pl, const Pipe& Pin, float* etab, float* efin,
                                           int q, int lane, int SH) {
  const Pipe P = Pin;  // in registers from here on
  const int m = 32 * q + lane;
  const uint32_t trow = P.tm + ((uint32_t)(32 * q) << 16);
  const int look = P.S > 2 ? 2 : P.S - 1;
  const bool fp4l = a.r_fmt == DSMOE_FMT_FP4;
  const bool w2_aligned = (a.row0 & 127) == 0;  // every w2 stage is then one FP8 scale segment
  int nseg = 0, n4 = 0, cur_g = -1, seg_ti = 0, unit = 0, gi = 0;
  uint32_t e4 = 0u;  // phase (bit 2 par + x) of each FP4 unit accumulator's barrier
  bool open = false, live = true;
  float acc[MAXB];
  Cur sf;  // runs ahead over the routed stages: FP4 scale factors of a stage into tensor memory
  sf.k = 4;
  auto store_sf = [&]() {
    const int slot = sf.g % P.S;
    if ((sf.k & 1) && pwait(a, pl, &P.full[slot], (sf.g / P.S) & 1)) {
      const uint4 v = *reinterpret_cast<const uint4*>(P.ring + (size_t)slot * STAGE + SA + SB + 16 * lane);
      tm_st4(trow + TM_SFA + 4 * slot, v.x, v.y, v.z, v.w);
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&P.sfr[slot]);
    }
    sf.next(P);
  };
  // A closed FP8 segment: its accumulator times the segment's scale (table entry ti) into acc.
  auto close_seg = [&](const float* tab, int ti) {
    const int slot_a = nseg & (NACC8 - 1);
    const bool got = pwait(a, pl, &P.accf[slot_a], (nseg / NACC8) & 1);
    ++nseg;
    if (!got) return;
    fence_after();
    float d[16];
    tm_ld16(trow + 16 * slot_a, d);
    fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&P.accr[slot_a]);
    const float s = tab[ti];
#pragma unroll
    for (int t = 0; t < MAXB; ++t) acc[t] = fmaf(d[t] + d[8 + t] * kLoInv, s, acc[t]);
  };
  // Two consecutive closed segments (tables entries ti0, ti1): one tensor-memory wait for both, the
  // same additions in the same order as two single closes.
  auto close_seg2 = [&](const float* tab, int ti0, int ti1) {
    const int sa = nseg & (NACC8 - 1), sb = (nseg + 1) & (NACC8 - 1);
    const bool ga = pwait(a, pl, &P.accf[sa], (nseg / NACC8) & 1);
    const bool gb = ga && pwait(a, pl, &P.accf[sb], ((nseg + 1) / NACC8) & 1);
    nseg += 2;
    if (!gb) return;
    fence_after();
    float d0[16], d1[16];
    tm_ld16x2(trow + 16 * sa, trow + 16 * sb, d0, d1);
    fence_before();
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&P.accr[sa]);
      mbar_arrive(&P.accr[sb]);
    }
    const float s0 = tab[ti0], s1 = tab[ti1];
#pragma unroll
    for (int t = 0; t < MAXB; ++t) {
      acc[t] = fmaf(d0[t] + d0[8 + t] * kLoInv, s0, acc[t]);
      acc[t] = fmaf(d1[t] + d1[8 + t] * kLoInv, s1, acc[t]);
    }
  };
  // Control flow here is the same in all four warps whatever happens (named barriers below): after an
  // expired wait the loop keeps walking the stream but skips the waits and the work.
  int g = 0;
  for (int k = 0; k < 4; ++k) {
    if (k == 1) {  // the routed units exist once the plan is published
      if (m == 0) wait_ready(a, pl, P.rdy);
      named_bar_sync(2, 128);
      if (fp4l) sf.start(P, 1, g);
    }
    const bool f4 = (k & 1) && fp4l, w13 = k < 2;
    const int nu = P.ucnt[k];
    for (int u = 0; u < nu; ++u) {
      const Unit U = P.units[k * UMAX + u];
      const int gi0 = gi;  // stream index (after the shared w1|w3 phase) of the unit's first stage
      if (k >= 1) gi += U.n;
      float* tab = etab + (unit & 1) * 256;
#pragma unroll
      for (int t = 0; t < MAXB; ++t) acc[t] = 0.f;
      live = !bar_any(2, 128, pl.abort != 0);  // the same in all four warps: a unit after a failure is skipped
      if (!f4 && live) {  // the unit's FP8 scale table (4 floats per block), read once by the four warps
        const uint8_t* st = w13 ? (U.slot >= 0 ? a.r13 + (long long)U.expert * a.r_eb13 + a.r_d13 : a.s13 + a.s_d13)
                                : (U.slot >= 0 ? a.r2 + (long long)U.expert * a.r_eb2 + a.r_d2 : a.s2 + a.s_d2);
        const float* src = reinterpret_cast<const float*>(st) + (long long)(U.tile * (w13 ? a.KB1 : a.KB2) + U.j0) * 4;
        for (int i = m; i < 4 * U.n; i += 128) tab[i] = __ldg(src + i);
        named_bar_sync(2, 128);
      }
      // w1|w3 rows: w1 rows 0..63, w3 rows 64..127 of the tile; the scale of this row's 128-row block
      int toff = 0;
      if (w13) {
        const int mat = m >> 6, r = 64 * U.tile + (m & 63);
        toff = 2 * mat + (((a.row0 + r) >> 7) != ((a.row0 + 64 * U.tile) >> 7) ? 1 : 0);
      }
      for (int j = U.j0; j < U.j0 + U.n; ++j, ++g) {
        const bool last = j == U.j0 + U.n - 1;
        // Never wait ahead on a w2 stage while this CTA still owes w1|w3 partials: w2 stages wait for
        // every CTA's w1|w3 work of their slot (so that wait could depend on this very epilogue).
        if (fp4l)
          while (sf.valid() && sf.g <= g + look && (sf.k < 2 || k >= 2)) store_sf();
        if (f4) {
          if (last) {  // the unit's accumulators of both MMA issuers (issuer x holds the stages of stream parity x)
            const int par = n4 & 1;
            float hi[MAXB], lo[MAXB];
#pragma unroll
            for (int t = 0; t < MAXB; ++t) hi[t] = lo[t] = 0.f;
#pragma unroll
            for (int x = 0; x < NISS; ++x) {
              if (a.ar_world <= 1 ? (U.n >= 2 || (gi0 & 1) == x) : x == 0) {
                const int bx = 2 * par + x;
                if (pwait(a, pl, &P.a4f[bx], (e4 >> bx) & 1u)) {
                  fence_after();
                  float d[16];
                  tm_ld16(trow + TM_ACC4 + 16 * bx, d);
                  fence_before();
                  __syncwarp();
                  if (lane == 0) mbar_arrive(&P.a4r[bx]);
#pragma unroll
                  for (int t = 0; t < MAXB; ++t) {
                    hi[t] += d[t];
                    lo[t] += d[8 + t];
                  }
                }
                e4 ^= 1u << bx;
              }
            }
#pragma unroll
            for (int t = 0; t < MAXB; ++t) acc[t] = hi[t] + lo[t] * kLoInv;
            ++n4;
          }
        } else if (w13 || w2_aligned) {  // the stage is exactly one scale segment
          if (!fp4l && !last) {  // this stage and the next together (the SF look-ahead is FP4-only)
            close_seg2(tab, 4 * (j - U.j0) + toff, 4 * (j + 1 - U.j0) + toff);
            ++j;
            ++g;
          } else {
            close_seg(tab, 4 * (j - U.j0) + toff);
          }
        } else {  // w2 of a slice that starts inside a 128-row block: the same segments as the MMA issuer
          const int nk = ksteps(a.I_loc, k, j);
          for (int qk = 0; qk < nk; ++qk) {
            const int gk = seg_key(a.row0, k, j, qk);
            if (!open || gk != cur_g) {
              if (open) close_seg(tab, seg_ti);
              open = true;
              cur_g = gk;
              // scale table entry: .x / .y of the block where the segment starts
              seg_ti = 4 * (j - U.j0) + (gk != ((a.row0 + 128 * j) >> 7) ? 1 : 0);
            }
          }
          if (last || seg_next(a.row0, k, j) != cur_g) {
            close_seg(tab, seg_ti);
            open = false;
          }
        }
      }
      // the unit's partial: 128 rows x 8 token columns, at this CTA's contributor index of the tile
      const int si = U.slot < 0 ? SH : U.slot;
      float* dst;
      if (w13) {
        dst = a.p13 + (((long long)si * a.P1 + U.tile) * MAXC + U.jc) * 1024;
#pragma unroll
        for (int t = 0; t < MAXB; ++t) acc[t] *= pl.xscale[t];
      } else {
        dst = a.p2 + (((long long)U.tile * a.slot_cap + si) * MAXC + U.jc) * 1024;
#pragma unroll
        for (int t = 0; t < MAXB; ++t) acc[t] *= (U.slot >= 0 && live ? pl.w[U.slot][t] : 1.0f) * (1.0f / kHScale);
      }
      if (live && !pl.abort && !(w13 && U.j0 == 0)) {  // (a w1|w3 tile's finisher keeps its own in registers)
        float4* d4 = reinterpret_cast<float4*>(dst + m * 8);
        d4[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        if (a.B > 4) d4[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
      }
      named_bar_sync(2, 128);
      // A w1|w3 tile is finished by the CTA holding its first blocks: in that CTA's range they come
      // last, while every other contributor holds the tile's later blocks at the start of its own
      // range. At N = 1 an output tile is finished by its designated CTA once the stream is done (see
      // below); at N > 1 by its last contributor's finisher warp. Units that cannot finish anything only
      // add their count (release: this CTA's partial, ordered by the barrier) and go on.
      const bool may_finish = w13 ? U.j0 == 0 : a.ar_world > 1;
      if (m == 0) {
        int fk = 0;  // what this CTA finishes: 1 a w1|w3 tile
        if (live && !pl.abort) {
          unsigned long long* cnt = w13 ? pl.cnt13 + (long long)si * a.P1 + U.tile : pl.cnt2 + U.tile;
          const unsigned long long total = w13 ? (unsigned long long)a.KB1 : (unsigned long long)((pl.nr + 1) * a.KB2);
          if (!may_finish) {
            red_add_release(cnt, (unsigned long long)U.n);
          } else if (w13) {
            // this CTA finishes the tile: it waits for the other contributors' counts (its own partial
            // stays in registers and is never counted), then acquires their partials (bounded wait)
            const unsigned long long others = total - (unsigned long long)U.n;
            const uint64_t t0 = globaltimer_ns();
            unsigned long long c;
            while ((c = ld_relaxed64(cnt)) < others) {
              if (ld_relaxed32(a.status) != 0u || globaltimer_ns() - t0 > kWait) {
                atomicOr(a.status, ST_CNT);
                pl.abort = 1;
                break;
              }
            }
            fence_acq_rel_gpu();
            if (c == others) {
              fk = 1;
            } else if (c > others) {
              atomicOr(a.status, ST_CNT);
              pl.abort = 1;
            }
          } else {
            // release: the partial of all 128 threads (ordered by the barrier); acquire: the other
            // contributors' partials once the count is complete
            const unsigned long long c = atom_add_acq_rel(cnt, (unsigned long long)U.n) + (unsigned long long)U.n;
            if (c == total) {  // N > 1: the exchange of the output tile runs on this CTA's finisher warp
              const int tail = *P.qtail;
              P.queue[tail % QCAP] = U.tile;
              __threadfence_block();
              *P.qtail = tail + 1;
            } else if (c > total) {
              atomicOr(a.status, ST_CNT);
              pl.abort = 1;
            }
          }
        }
        pl.efl = fk;
      }
      if (may_finish) {
        named_bar_sync(2, 128);
        if (*reinterpret_cast<volatile int*>(&pl.efl) == 1)
          epi_finish_w13(a, pl, U.slot < 0 ? 0 : 1, si, U.tile, U.tile_id, U.jc, acc, m, efin);
      }
      ++unit;
    }
  }
  // N = 1: the output tiles designated to this CTA (tile mt to CTA floor(mt G / MT2), at most one each
  // while MT2 <= G), each once all its (nr + 1) KB2 stage contributions are counted (bounded wait).
  if (a.ar_world <= 1) {
    const int G = gridDim.x;
    const int c = blockIdx.x;
    for (int mt = (int)(((unsigned)c * (unsigned)a.MT2 + (unsigned)G - 1u) / (unsigned)G);
         mt < a.MT2 && (int)((unsigned)mt * (unsigned)G / (unsigned)a.MT2) == c; ++mt) {
      named_bar_sync(2, 128);
      if (m == 0) {
        int go = 0;
        if (!pl.abort) {
          const unsigned long long total = (unsigned long long)((pl.nr + 1) * a.KB2);
          const uint64_t t0 = globaltimer_ns();
          while (ld_relaxed64(pl.cnt2 + mt) < total) {
            if (ld_relaxed32(a.status) != 0u || globaltimer_ns() - t0 > kWait) {
              atomicOr(a.status, ST_CNT);
              pl.abort = 1;
              break;
            }
          }
          fence_acq_rel_gpu();  // acquire: every contributor's partial
          go = pl.abort ? 0 : 1;
        }
        pl.efl = go;
      }
      named_bar_sync(2, 128);
      if (*reinterpret_cast<volatile int*>(&pl.efl) == 1) epi_finish_w2(a, pl, mt, SH, m, reinterpret_cast<int*>(efin + 2 * 64 * 8));
    }
  }
  named_bar_sync(2, 128);
  if (m == 0) {
    __threadfence_block();
    *P.edone = 1;
  }
}

// The units of kind k for this CTA, one per lane of the calling warp (all 32 lanes call): unit u is
// this CTA's part of the u-th tile its stage range touches.
__device__ __noinline__ void build_units(const TcArgs& a, const TcPlan& pl, int nr, int k, Unit* out, int* cnt,
                                         unsigned* status, int lane) {
  Split sp;
  const int G = gridDim.x, per = k < 2 ? a.P1 : a.MT2, spt = k < 2 ? a.KB1 : a.KB2;
  const int tiles = (k & 1) ? nr * per : per;
  sp.init(tiles * spt, spt, G);
  const int lo = sp.lo(blockIdx.x), hi = sp.hi(blockIdx.x);
  const int t0 = lo / spt, nu = hi > lo ? (hi - 1) / spt - t0 + 1 : 0;
  if (nu > UMAX) {
    if (lane == 0) {
      atomicOr(status, ST_PLAN);
      *cnt = 0;
    }
    return;
  }
  for (int u = lane; u < nu; u += 32) {
    const int tid_ = t0 + u, s = max(lo, tid_ * spt), e = min(hi, (tid_ + 1) * spt);
    Unit U;
    U.kind = (short)k;
    U.slot = (short)((k & 1) ? tid_ / per : -1);
    U.tile = (short)((k & 1) ? tid_ - U.slot * per : tid_);
    U.j0 = (short)(s - tid_ * spt);
    U.n = (short)(e - s);
    U.jc = (short)(blockIdx.x - sp.owner(tid_ * spt));
    U.expert = (k & 1) ? pl.expert[U.slot] : 0;
    U.tile_id = tid_;
    out[u] = U;
  }
  if (lane == 0) *cnt = nu;
}

// ---- the peer all-reduce of eight consecutive 16-row tiles (one 128-row output tile) by one warp:
// every tile's words go to every peer first, then all tiles of all peers are polled together.
// Same slots, epochs and words as ll_allreduce_tile (exchange.cuh), so both share one comm.
__device__ __noinline__ bool ll_allreduce_tiles8(unsigned long long* const* slots, int W, int r, int NTt, int nt0, int B,
                                                unsigned ep, float4 (&s4)[8], int lane, uint64_t limit_ns) {
  bool ok = true;
  if (2 * (lane & 3) < B) {
    const bool one = B == 1;
    const int par = (int)(ep & 1u);
    for (int d = 1; d < W; ++d) {
      const int q = r + d < W ? r + d : r + d - W;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        unsigned long long* p = slots[q] + ar_slot(par, r, W, NTt, nt0 + u, lane);
        st_ll2(p, ll_word(s4[u].x, ep), ll_word(one ? s4[u].z : s4[u].y, ep));
        if (!one) st_ll2(p + 2, ll_word(s4[u].z, ep), ll_word(s4[u].w, ep));
      }
    }
    float4 tot[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) tot[u] = make_float4(0.f, 0.f, 0.f, 0.f);
    // ranks in order: the same bits on every rank
    const uint64_t t0 = globaltimer_ns();
    for (int q = 0; q < W && ok; ++q) {
      if (q == r) {
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const float4 v = one ? make_float4(s4[u].x, 0.f, s4[u].z, 0.f) : s4[u];
          tot[u].x += v.x;
          tot[u].y += v.y;
          tot[u].z += v.z;
          tot[u].w += v.w;
        }
        continue;
      }
      unsigned got = 0u;
      float4 v[8];
      while (got != 0xFFu) {
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (!((got >> u) & 1u)) {
            const unsigned long long* p = slots[r] + ar_slot(par, q, W, NTt, nt0 + u, lane);
            unsigned long long x0, x1, x2 = 0ull, x3 = 0ull;
            ld_ll2(p, x0, x1);
            if (!one) ld_ll2(p + 2, x2, x3);
            const bool here = (unsigned)(x0 >> 32) == ep && (unsigned)(x1 >> 32) == ep &&
                              (one || ((unsigned)(x2 >> 32) == ep && (unsigned)(x3 >> 32) == ep));
            if (here) {
              v[u] = one ? make_float4(__uint_as_float((unsigned)x0), 0.f, __uint_as_float((unsigned)x1), 0.f)
                         : make_float4(__uint_as_float((unsigned)x0), __uint_as_float((unsigned)x1),
                                       __uint_as_float((unsigned)x2), __uint_as_float((unsigned)x3));
              got |= 1u << u;
            }
          }
        if (got != 0xFFu && globaltimer_ns() - t0 > limit_ns) {
          ok = false;
          break;
        }
      }
      if (!ok) break;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        tot[u].x += v[u].x;
        tot[u].y += v[u].y;
        tot[u].z += v[u].z;
        tot[u].w += v[u].w;
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) s4[u] = tot[u];
  }
  return __all_sync(0xffffffffu, ok);
}

// ---- warp 3: finisher (N > 1). Sums a finished output tile's partials in contributor order and runs
// its peer exchange; at N = 1 the epilogue finishes every tile itself.
// Loads the sum of a tile's partials ([MAXC][128 rows][8]) for rows 4 lane .. 4 lane + 3, B tokens,
// into fin[128][8]. The partials form a list of nb <= 8 entries in summation order: entry i is slot
// s = l0 + i (the shared slot SH once s >= nr), its partials at base + slot * estride, and lane i
// holds its count. The list is walked as one flat sequence, CAP partials at a time with all their
// loads in flight, so a tile costs one memory round trip per CAP partials whatever its slots.
template <int CAP, bool WIDE>
__device__ __forceinline__ void sum_partials_t(const float* base, long long estride, int l0, int nr, int SH,
                                               const int (&pre)[9], float (&s)[4][MAXB], int lane) {
  const int total = pre[8];
  for (int f0 = 0; f0 < total; f0 += CAP) {
    uint4 v[CAP][4][WIDE ? 2 : 1];
#pragma unroll
    for (int p = 0; p < CAP; ++p) {
      const int f = f0 + p;
      if (f < total) {
        int li = 0, at = 0;
#pragma unroll
        for (int q = 1; q < 8; ++q)
          if (f >= pre[q]) {
            li = q;
            at = pre[q];
          }
        const int sl = l0 + li < nr ? l0 + li : SH;
        const float* src = base + sl * estride + (f - at) * 1024 + 4 * lane * 8;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          v[p][r][0] = ld_cg16(src + r * 8);
          if (WIDE) v[p][r][WIDE ? 1 : 0] = ld_cg16(src + r * 8 + 4);
        }
      }
    }
#pragma unroll
    for (int p = 0; p < CAP; ++p)
      if (f0 + p < total)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          s[r][0] += __uint_as_float(v[p][r][0].x);
          s[r][1] += __uint_as_float(v[p][r][0].y);
          s[r][2] += __uint_as_float(v[p][r][0].z);
          s[r][3] += __uint_as_float(v[p][r][0].w);
          if (WIDE) {
            s[r][4] += __uint_as_float(v[p][r][WIDE ? 1 : 0].x);
            s[r][5] += __uint_as_float(v[p][r][WIDE ? 1 : 0].y);
            s[r][6] += __uint_as_float(v[p][r][WIDE ? 1 : 0].z);
            s[r][7] += __uint_as_float(v[p][r][WIDE ? 1 : 0].w);
          }
        }
  }
}
__device__ __noinline__ void sum_partials(const float* base, long long estride, int l0, int nr, int SH, int nb,
                                          int cnt_lane, int B, float* fin, int lane) {
  int pre[9];  // first flat index of each list entry (entries past the list start at the end)
  pre[0] = 0;
#pragma unroll
  for (int q = 0; q < 8; ++q) pre[q + 1] = pre[q] + (q < nb ? __shfl_sync(0xffffffffu, cnt_lane, q) : 0);
  float s[4][MAXB];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int t = 0; t < MAXB; ++t) s[r][t] = 0.f;
  if (B > 4)
    sum_partials_t<3, true>(base, estride, l0, nr, SH, pre, s, lane);
  else
    sum_partials_t<6, false>(base, estride, l0, nr, SH, pre, s, lane);
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int t = 0; t < MAXB; ++t) fin[(4 * lane + r) * 8 + t] = s[r][t];
  __syncwarp();
}

// Output tile m finished: y rows [128 m, 128 m + 128) = sum over the routed slots (in order) and the
// shared expert of their partials; at N > 1 summed over the ranks through the peer exchange.
__device__ __noinline__ void finish_w2(const TcArgs& a, TcPlan& pl, int m, int SH, float* fin, int lane) {
  const int nl = pl.nr + 1;
  bool ok = true;
  // partials of slots in order, in batches that fit the local lists
  float acc[4][MAXB];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int t = 0; t < MAXB; ++t) acc[r][t] = 0.f;
  const int nr = pl.nr;
  for (int l0 = 0; l0 < nl; l0 += 8) {
    // lane i < 8 counts the contributors of list entry i (slot l0 + i; the shared expert last)
    const int nb = min(8, nl - l0), s = l0 + lane;
    const int cnt = lane < nb ? contrib_count(pl.wk.sp[s < nr ? 3 : 2], s < nr ? s * a.MT2 + m : m) : 0;
    sum_partials(a.p2 + (long long)m * a.slot_cap * MAXC * 1024, (long long)MAXC * 1024, l0, nr, SH, nb, cnt, a.B, fin,
                 lane);
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int t = 0; t < MAXB; ++t) acc[r][t] += fin[(4 * lane + r) * 8 + t];
    __syncwarp();
  }
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int t = 0; t < MAXB; ++t) fin[(4 * lane + r) * 8 + t] = acc[r][t];
  __syncwarp();
  if (a.ar_world > 1) {
    // eight 16-row tiles through the exchange: every tile's words sent first, then all polled
    const int t0 = 2 * (lane & 3);
    float4 s4[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int r = 16 * u + (lane >> 2);
      s4[u] = make_float4(fin[r * 8 + t0], fin[r * 8 + t0 + 1], fin[(r + 8) * 8 + t0], fin[(r + 8) * 8 + t0 + 1]);
    }
    ok = ll_allreduce_tiles8(a.ar_slots, a.ar_world, a.ar_rank, a.H / 16, 8 * m, a.B, pl.ar_epoch, s4, lane, kPeerWait);
    __syncwarp();
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int r = 16 * u + (lane >> 2);
      if (t0 < a.B) {
        fin[r * 8 + t0] = s4[u].x;
        fin[r * 8 + t0 + 1] = s4[u].y;
        fin[(r + 8) * 8 + t0] = s4[u].z;
        fin[(r + 8) * 8 + t0 + 1] = s4[u].w;
      }
    }
    __syncwarp();
    if (!ok && lane == 0) atomicOr(a.status, ST_PEER);
  }
  // y rows 4 lane .. 4 lane + 3 of every token
  for (int t = 0; t < a.B; ++t) {
    float v[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) v[r] = ok ? fin[(4 * lane + r) * 8 + t] : __int_as_float(0x7FC00000);
    const long long o = (long long)t * a.H + 128 * m + 4 * lane;
    if (a.y_f32) {
      *reinterpret_cast<float4*>(reinterpret_cast<float*>(a.y) + o) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
      const __nv_bfloat162 p0 = __floats2bfloat162_rn(v[0], v[1]), p1 = __floats2bfloat162_rn(v[2], v[3]);
      *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(a.y) + o) =
          make_uint2(*reinterpret_cast<const uint32_t*>(&p0), *reinterpret_cast<const uint32_t*>(&p1));
    }
  }
  __syncwarp();
}

__device__ __noinline__ void role_finisher(const TcArgs& a, TcPlan& pl, const Pipe& Pin, float* fin, int lane, int SH) {
  const Pipe P = Pin;
  int head = 0;
  uint64_t t0 = globaltimer_ns();
  while (true) {
    int job = -1;
    if (lane == 0) {
      while (true) {
        if (head < *P.qtail) {
          job = P.queue[head % QCAP];
          break;
        }
        if (*P.edone && head >= *P.qtail) break;
        if (pl.abort) break;
        backoff();
        if (globaltimer_ns() - t0 > 4 * kWait) {  // the epilogue has not finished in time
          atomicOr(a.status, ST_CNT);
          pl.abort = 1;
          break;
        }
      }
    }
    job = __shfl_sync(0xffffffffu, job, 0);
    if (job < 0) break;
    ++head;
    t0 = globaltimer_ns();
    fence_acq_rel_gpu();  // acquire: the other CTAs' partials
    finish_w2(a, pl, job, SH, fin, lane);
  }
}

// ------------------------------------------------------------------ the kernel
__global__ void __launch_bounds__(NT, 1) moe_tc_kernel(const __grid_constant__ TcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const TcSmem L = tc_smem(a.H, a.S, a.E, a.B);
  Pipe P;
  P.S = a.S;
  P.ring = sm + L.ring;
  P.xb = sm + L.xb;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L.bars);
  P.full = bars;
  P.empty = bars + a.S;
  P.sfr = bars + 2 * a.S;
  P.accf = bars + 3 * a.S;
  P.accr = P.accf + NACC8;
  P.a4f = P.accr + NACC8;
  P.a4r = P.a4f + 2 * NISS;
  P.mdone = P.a4r + 2 * NISS;
  P.rdy = P.mdone + NISS;
  TcPlan& pl = *reinterpret_cast<TcPlan*>(sm + L.plan);
  unsigned* emask = reinterpret_cast<unsigned*>(sm + L.emask);
  float* etab = reinterpret_cast<float*>(sm + L.etab);
  float* fin = reinterpret_cast<float*>(sm + L.fin);
  float* efin = reinterpret_cast<float*>(sm + L.efin);
  P.queue = reinterpret_cast<int*>(sm + L.queue);
  P.qtail = reinterpret_cast<volatile int*>(P.queue + QCAP);
  P.edone = P.qtail + 1;
  P.issued = P.qtail + 2;
  Unit* units = reinterpret_cast<Unit*>(sm + L.units);
  int* ucnt = reinterpret_cast<int*>(units + 4 * UMAX);
  P.units = units;
  P.ucnt = ucnt;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + L.misc);
  unsigned long long* gbase_s = reinterpret_cast<unsigned long long*>(sm + L.misc + 8);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, SH = a.slot_cap - 1;

  if (tid == 0) {
    // This CTA's router rows and the router biases into L2 now (constant data): the router and the
    // plan then read them at L2 latency.
    {
      const int r0 = (int)((unsigned)a.E * (unsigned)blockIdx.x / (unsigned)G);
      const int r1 = (int)((unsigned)a.E * (unsigned)(blockIdx.x + 1) / (unsigned)G);
      if (r1 > r0) prefetch_l2(a.wg + (long long)r0 * a.H, (uint32_t)((r1 - r0) * a.H * 4));
      if (a.bias != nullptr && ((uintptr_t)a.bias & 15) == 0 && (a.E & 3) == 0) prefetch_l2(a.bias, (uint32_t)(a.E * 4));
    }
    for (int s = 0; s < a.S; ++s) {
      mbar_init(&P.full[s], 1);
      mbar_init(&P.empty[s], 1);
      mbar_init(&P.sfr[s], 4);
    }
    for (int i = 0; i < NACC8; ++i) {
      mbar_init(&P.accf[i], 1);
      mbar_init(&P.accr[i], 4);
    }
    for (int i = 0; i < 2 * NISS; ++i) {
      mbar_init(&P.a4f[i], 1);
      mbar_init(&P.a4r[i], 4);
    }
    for (int i = 0; i < NISS; ++i) mbar_init(&P.mdone[i], 1);
    mbar_init(P.rdy, 1);
    ucnt[1] = ucnt[3] = 0;
    pl.nr = 0;
    pl.efl = 0;
    pl.wk.init(a, 0);  // the shared expert's splits now; the routed ones once the plan is known
    pl.tag = 0u;
    pl.ar_epoch = 0u;
    pl.ready = 0;
    pl.abort = 0;
    *P.qtail = 0;
    *P.edone = 0;
    *P.issued = 0;
    fence_mbar_init();
  }
  if (warp == 0) {  // the shared expert's units do not depend on routing: listed now, so its weights stream at once
    build_units(a, pl, 0, 0, units, &ucnt[0], a.status, lane);
    build_units(a, pl, 0, 2, units + 2 * UMAX, &ucnt[2], a.status, lane);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)), "r"(TM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  P.tm = *tslot;

  if (warp == 0) {
    // Constant weights only: with a programmatic dependent launch this overlaps the previous kernel.
    if (lane == 0) role_producer(a, pl, P);
  } else {
    // Past this point the previous kernel in the stream has completed (tokens, workspace, epoch).
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int t7 = tid - 32;
    if (t7 == 0) {
      const unsigned long long c = ld_relaxed64(a.gbar);
      const unsigned long long gb = c - c % (unsigned long long)G;
      *gbase_s = gb;
      pl.tag = (unsigned)((gb / (unsigned long long)G) % 0xFFFFFFFFull) + 1u;
      {
        unsigned long long* mine = a.cnt + (long long)(pl.tag & 1u) * a.cnt_words;
        unsigned long long* next = a.cnt + (long long)((pl.tag & 1u) ^ 1u) * a.cnt_words;
        pl.cnt13 = mine;
        pl.cnt2 = mine + a.slot_cap * a.P1;
        pl.sdone = pl.cnt2 + a.MT2;
        // the previous launch (parity of the next one) has completed: its counters go back to zero
        for (int i = blockIdx.x; i < a.cnt_words; i += G) next[i] = 0ull;
      }
      pl.ar_epoch = a.ar_world > 1 ? *(volatile unsigned*)a.ar_ctl + 1u : 0u;
      if (ld_relaxed32(a.status) != 0u) pl.abort = 1;  // an earlier call gave up: stop until reset
      fence_acq_rel_gpu();
      asm volatile("red.relaxed.gpu.global.add.u64 [%0], 1;" ::"l"(a.gbar) : "memory");  // read the epoch
      asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    }
    // The B tile first (its first barrier also publishes the tag): the MMA issuer starts on the
    // shared expert as soon as it exists, while warps 2-7 compute this CTA's router rows and warps
    // 2-3 then gather every CTA's rows into the plan.
    build_xb(a, P.xb, pl, fin, t7);
    const bool ok0 = !bar_any(1, 224, pl.abort != 0);
    if (warp == 1) {
      if (lane == 0) role_mma(a, pl, P, 0);
    } else {
      if (warp >= 4) {  // B-side scale factors of the block-scaled MMA: 1.0 for every row and group
        tm_st4(P.tm + ((uint32_t)(32 * (warp - 4)) << 16) + TM_SFB, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu);
        fence_before();
      }
      if (ok0) router_rows(a, pl, warp - 2, 6, lane, reinterpret_cast<double*>(efin));
      if (warp >= 4) {
        role_epilogue(a, pl, P, etab, efin, warp - 4, lane, SH);
      } else {
        const int tp = tid - 64;
        float* scr = reinterpret_cast<float*>(sm + L.scr);
        const bool ok = ok0 && make_plan(a, pl, scr, scr + a.B * a.E, emask, tp);
        // The routed units follow from the plan. Without one (a failed set-up) every role walks the
        // shared expert's stages only, and skips them (the call has already given up).
        const int nr = ok ? pl.nr : 0;
        build_units(a, pl, nr, warp == 2 ? 1 : 3, units + (warp == 2 ? 1 : 3) * UMAX, &ucnt[warp == 2 ? 1 : 3], a.status,
                    lane);
        named_bar_sync(BAR_PLAN, PT);
        if (warp == 2) {
          if (lane == 0) {  // the routed splits (the shared ones, read meanwhile, stay as they are)
            pl.nr = nr;
            pl.wk.nr = nr;
            pl.wk.sp[1].init(nr * a.P1 * a.KB1, a.KB1, G);
            pl.wk.sp[3].init(nr * a.MT2 * a.KB2, a.KB2, G);
            __threadfence_block();
            pl.ready = 1;
            mbar_arrive(P.rdy);
          }
          if (lane == 0) role_hcopy(a, pl, P, SH);
        } else if (a.ar_world > 1) {
          role_finisher(a, pl, P, fin, lane, SH);
        } else {  // N = 1: the epilogue finishes every tile; this warp is the second MMA issuer
          if (lane == 0) role_mma(a, pl, P, 1);
        }
      }
    }
  }
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(P.tm), "r"(TM_COLS) : "memory");
  if (blockIdx.x == 0 && tid == 0 && a.ar_world > 1) {
    // every CTA has read the exchange epoch (one arrival each at its start): publish the next one
    const uint64_t t0 = globaltimer_ns();
    while ((long long)(ld_relaxed64(a.gbar) - (*gbase_s + (unsigned long long)G)) < 0) {
      if (globaltimer_ns() - t0 > kWait) {
        atomicOr(a.status, ST_CNT);
        break;
      }
    }
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(a.ar_ctl), "r"(pl.ar_epoch) : "memory");
  }
  // A call that gave up (here or in an earlier call on this workspace) leaves NaN in its share of y
  // (128-row tiles m = cta + G j) rather than stale memory.
  if (ld_relaxed32(a.status) != 0u) {
    for (int m = blockIdx.x; m < a.MT2; m += G)
      for (int i = tid; i < 128 * a.B; i += NT) {
        const long long o = (long long)(i >> 7) * a.H + 128 * m + (i & 127);
        if (a.y_f32)
          reinterpret_cast<float*>(a.y)[o] = __int_as_float(0x7FC00000);
        else
          reinterpret_cast<__nv_bfloat16*>(a.y)[o] = __ushort_as_bfloat16((unsigned short)0x7FC0);
      }
  }
}

}  // namespace tc

// ------------------------------------------------------------------ host side
// Workspace of the tensor-core path (laid out for 8 tokens whatever the call's batch): the grid
// counter and the status word at the same offsets as the persistent fragment-layout path, then the
// tagged router partials and counters (cleared together by dsmoe_moe_check), then partials and h.
TcScratch tc_scratch(const dsmoe_layer_t* L) {
  TcScratch f{};
  const int P1 = (L->inter_local + 63) / 64, KB2 = (L->inter_local + 127) / 128, MT2 = L->hidden / 128;
  f.slot_cap = tc::MAXB * L->topk + 1;
  auto al = [](size_t v) { return (v + 255) & ~size_t(255); };
  size_t o = 0;
  f.gbar = o; o += al(8);
  f.status = o; o += al(4);
  f.rl = o; o += al((size_t)tc::MAXB * L->n_experts * 4 * 16);
  f.cnt_words = f.slot_cap * P1 + MT2 + f.slot_cap;
  f.cnt = o; o += al((size_t)2 * f.cnt_words * 8);  // one counter set per launch parity
  f.counters_end = o;
  f.p13 = o; o += al((size_t)f.slot_cap * P1 * tc::MAXC * 4096);
  f.p2 = o; o += al((size_t)MT2 * f.slot_cap * tc::MAXC * 4096);
  f.hb = o; o += al((size_t)f.slot_cap * KB2 * 2048);
  f.total = o;
  return f;
}

namespace {

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::mutex g_tc_mu;

struct TcKey {
  const void* p[4];
  int H, I_loc, row0, E, fmt;
  bool operator==(const TcKey& o) const {
    return p[0] == o.p[0] && p[1] == o.p[1] && p[2] == o.p[2] && p[3] == o.p[3] && H == o.H && I_loc == o.I_loc &&
           row0 == o.row0 && E == o.E && fmt == o.fmt;
  }
};
struct TcMaps {
  TcKey key;
  CUtensorMap r13, r2, s13, s2;
  bool used;
};
constexpr int kMapCache = 512;
TcMaps g_maps[kMapCache];
int g_maps_next = 0;

int encode(CUtensorMap* m, bool fp4, int rank, const void* base, const cuuint64_t* dims, const cuuint64_t* strides,
           const cuuint32_t* box) {
  const cuuint32_t es[4] = {1, 1, 1, 1};
  const CUresult r = g_encode(m, fp4 ? CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B : CU_TENSOR_MAP_DATA_TYPE_UINT8, rank,
                              const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  DSMOE_REQUIRE(r == CUDA_SUCCESS, DSMOE_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return DSMOE_OK;
}

// An expert set's w1|w3 or w2 blocks as a 4-D tensor {K in a block (128), rows (128), block, expert}:
// one box is one contiguous block.
int encode_store(const dsmoe_store_t& st, int H, int I_loc, CUtensorMap* m13, CUtensorMap* m2) {
  const TcGeom g = tc_geom(st.fmt, H, I_loc + st.row0, st.row0, I_loc);
  const bool f4 = st.fmt == DSMOE_FMT_FP4;
  const cuuint32_t box[4] = {128, 128, 1, 1};
  const cuuint64_t d13[4] = {128, 128, (cuuint64_t)g.P1 * g.KB1, (cuuint64_t)st.n_experts};
  const cuuint64_t s13[3] = {(cuuint64_t)g.row_bytes, (cuuint64_t)g.blk, (cuuint64_t)st.w13_expert_bytes};
  int rc = encode(m13, f4, 4, st.w13, d13, s13, box);
  if (rc) return rc;
  const cuuint64_t d2[4] = {128, 128, (cuuint64_t)g.MT2 * g.KB2, (cuuint64_t)st.n_experts};
  const cuuint64_t s2[3] = {(cuuint64_t)g.row_bytes, (cuuint64_t)g.blk, (cuuint64_t)st.w2_expert_bytes};
  return encode(m2, f4, 4, st.w2, d2, s2, box);
}

int get_maps(const dsmoe_layer_t* L, TcMaps** out) {
  std::lock_guard<std::mutex> lk(g_tc_mu);
  if (!g_encode) {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return cuda_status("moe_tc: cuTensorMapEncodeTiled entry point");
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  TcKey k{{L->routed.w13, L->routed.w2, L->shared.w13, L->shared.w2}, L->hidden, L->inter_local,
          L->routed.row0, L->n_experts, L->routed.fmt};
  for (int i = 0; i < kMapCache; ++i)
    if (g_maps[i].used && g_maps[i].key == k) {
      *out = &g_maps[i];
      return DSMOE_OK;
    }
  TcMaps& m = g_maps[g_maps_next];
  g_maps_next = (g_maps_next + 1) % kMapCache;
  m.used = false;
  int rc = encode_store(L->routed, L->hidden, L->inter_local, &m.r13, &m.r2);
  if (!rc) rc = encode_store(L->shared, L->hidden, L->inter_local, &m.s13, &m.s2);
  if (rc) return rc;
  m.key = k;
  m.used = true;
  *out = &m;
  return DSMOE_OK;
}

struct TcDev {
  int sms = 0, optin = 0;
  bool attr = false;
  int pdl = -1;
};
TcDev g_tcdev[64];

}  // namespace

bool tc_supported(const dsmoe_layer_t* L, int B) {
  if (B < 1 || B > tc::MAXB || L->n_experts > tc::MAXE || L->hidden % 128 || L->hidden > 8192 ||
      L->inter_local % 32 || L->inter_local < 64 || L->inter_local > 8192 || L->topk > tc::MAXK)
    return false;
  if (L->routed.layout != DSMOE_LAYOUT_TC || L->shared.layout != DSMOE_LAYOUT_TC || L->shared.fmt != DSMOE_FMT_FP8 ||
      L->shared.n_experts != 1 || L->shared.row0 != L->routed.row0)
    return false;
  int dev = 0;
  cudaGetDevice(&dev);
  TcDev& d = g_tcdev[dev & 63];
  if (d.sms == 0) {
    cudaDeviceGetAttribute(&d.optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
  }
  // a CTA's router rows (E / SMs, rounded up) keep their quarter sums in the epilogue's scratch
  if ((L->n_experts + d.sms - 1) / d.sms * 4 * tc::MAXB * 8 > 2 * 64 * 8 * 4) return false;
  return tc::tc_smem(L->hidden, 3, L->n_experts, tc::MAXB).total <= (size_t)d.optin;
}

int launch_tc(const dsmoe_layer_t* L, const void* x, int B, const uint8_t* image_mask, void* y, int y_dtype,
              int64_t* idx, float* wt, float* scores, uint8_t* ws, cudaStream_t st, const PeerExchange* px) {
  int dev = 0;
  cudaGetDevice(&dev);
  TcDev& d = g_tcdev[dev & 63];
  TcMaps* maps = nullptr;
  int rc = get_maps(L, &maps);
  if (rc) return rc;
  const TcScratch f = tc_scratch(L);
  tc::TcArgs a{};
  a.tm_r13 = maps->r13;
  a.tm_r2 = maps->r2;
  a.tm_s13 = maps->s13;
  a.tm_s2 = maps->s2;
  a.H = L->hidden;
  a.I_loc = L->inter_local;
  a.row0 = L->routed.row0;
  a.E = L->n_experts;
  a.B = B;
  a.topk = L->topk;
  a.score_func = L->score_func;
  a.route_scale = L->route_scale;
  a.r_fmt = L->routed.fmt;
  const TcGeom gr = tc_geom(L->routed.fmt, L->hidden, L->inter_local + a.row0, a.row0, L->inter_local);
  const TcGeom gs = tc_geom(DSMOE_FMT_FP8, L->hidden, L->inter_local + a.row0, a.row0, L->inter_local);
  a.P1 = gr.P1;
  a.KB1 = gr.KB1;
  a.KB2 = gr.KB2;
  a.MT2 = gr.MT2;
  // as many ring stages as fit next to the B tile and the rest (at most MAXS)
  int S = tc::MAXS;
  while (S > 0 && tc::tc_smem(L->hidden, S, L->n_experts, B).total > (size_t)d.optin) --S;
  DSMOE_REQUIRE(S >= 3, DSMOE_ERR_UNSUPPORTED, "moe_tc: shared memory for %d stages only", S);
  a.S = S;
  a.slot_cap = f.slot_cap;
  a.wg = L->gate_w;
  a.bias = L->gate_bias;
  a.bias_vl = L->gate_bias_vl;
  a.image_mask = image_mask;
  a.x = (const __nv_bfloat16*)x;
  a.r13 = L->routed.w13;
  a.r2 = L->routed.w2;
  a.r_eb13 = L->routed.w13_expert_bytes;
  a.r_eb2 = L->routed.w2_expert_bytes;
  a.r_d13 = gr.d13;
  a.r_d2 = gr.d2;
  a.s13 = L->shared.w13;
  a.s2 = L->shared.w2;
  a.s_d13 = gs.d13;
  a.s_d2 = gs.d2;
  a.y = y;
  a.y_f32 = y_dtype == DSMOE_DTYPE_F32;
  a.idx = idx;
  a.wt = wt;
  a.scores = scores;
  a.gbar = (unsigned long long*)(ws + f.gbar);
  a.status = (unsigned*)(ws + f.status);
  a.rl = (unsigned long long*)(ws + f.rl);
  a.cnt = (unsigned long long*)(ws + f.cnt);
  a.cnt_words = f.cnt_words;
  a.p13 = (float*)(ws + f.p13);
  a.p2 = (float*)(ws + f.p2);
  a.hb = ws + f.hb;
  if (px && px->world > 1) {
    DSMOE_REQUIRE(px->hidden == L->hidden && px->world <= kMaxWorld && px->rank >= 0 && px->rank < px->world,
                  DSMOE_ERR_ARG, "moe_tc: exchange for hidden %d, world %d, rank %d", px->hidden, px->world, px->rank);
    a.ar_world = px->world;
    a.ar_rank = px->rank;
    a.ar_ctl = px->ctl;
    for (int q = 0; q < px->world; ++q) {
      DSMOE_REQUIRE(px->slots[q], DSMOE_ERR_ARG, "moe_tc: exchange slots of rank %d not mapped", q);
      a.ar_slots[q] = px->slots[q];
    }
  }
  const size_t smem = tc::tc_smem(L->hidden, S, L->n_experts, B).total;
  if (!d.attr) {
    if (cudaFuncSetAttribute(tc::moe_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, d.optin) != cudaSuccess)
      return cuda_status("moe_tc: set smem");
    d.attr = true;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(d.sms);
  cfg.blockDim = dim3(tc::NT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (d.pdl < 0) cudaStreamIsCapturing(st, &cap);
  const bool try_pdl = d.pdl == 1 || (d.pdl < 0 && cap == cudaStreamCaptureStatusNone);
  cfg.numAttrs = try_pdl ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, tc::moe_tc_kernel, a);
  if (try_pdl && d.pdl < 0) {
    if (e == cudaSuccess) {
      d.pdl = 1;
    } else {
      cudaGetLastError();
      d.pdl = 0;
      cfg.numAttrs = 1;
      e = cudaLaunchKernelEx(&cfg, tc::moe_tc_kernel, a);
    }
  }
  if (e != cudaSuccess) {
    set_error("moe_tc launch: %s", cudaGetErrorString(e));
    cudaGetLastError();
    return DSMOE_ERR_CUDA;
  }
  return DSMOE_OK;
}

}  // namespace dsmoe
