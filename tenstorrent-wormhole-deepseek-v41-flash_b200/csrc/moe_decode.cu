// Decode-regime MoE layer (1..64 tokens): fused dequant + tensor-core GEMV over resident experts.
//
// Reference path replaced: MoE.decode (dsv41/tt/moe.py:148-180) -- slot gather of the six host-
// chosen experts into concatenated buffers (dsv41/kernels/slot_cat.cpp:194-365), three matmuls,
// the Q20 SwiGLU kernel (dsv41/kernels/slot_cat.cpp:82-192) and the weighted combine -- and its
// multi-token form verify_batched (dsv41/tt/moe.py:202-241).
//
// Per step (after the router kernels, router.cu):
//   moe_w13_kernel  grid (inter_local/16 tiles, slots): one CTA streams one 16-row tile of w1 and
//                   of w3 for one slot (expert + up to 8 tokens), 8 warps split K, mma.sync
//                   m16n8k32 on the e4m3 weights (FP4 expanded to e4m3 in registers) against the
//                   tokens' e4m3 hi / lo terms, fp32 accumulation, per-block (FP8) or per-32 (FP4)
//                   scales applied to the fp32 partials; epilogue: clamp, SiLU(g)*u -> h as e4m3
//                   hi / lo rows in the order w2 reads.
//   moe_w2_kernel   grid hidden/16: one CTA owns 16 output rows for all slots and all tokens;
//                   warps split the (slot, K-chunk) items evenly; routing weight on the fp32
//                   partials; deterministic combine in smem.
// Both kernels are HBM-bound: every weight byte of the touched experts is read exactly once per
// step, with 16-byte streaming loads, 4 independent chunks in flight per warp.
#include "router.cuh"

namespace dsmoe {

struct DecodeArgs {
  int H, I_loc, E, B;
  int r_fmt;
  const uint8_t* r_w13;
  const uint8_t* r_w2;
  long long r_w13_eb, r_w2_eb;
  const uint8_t* s_w13;  // shared expert (FP8)
  const uint8_t* s_w2;
  const int* plan;
  const int* slot_expert;
  const int* slot_ntok;
  const int* slot_tok;
  const float* slot_wt;
  const uint8_t* xq;     // [B][2][H] e4m3 hi / lo token rows
  const float* xscale;   // [B]
  uint8_t* hq;           // [slots] h rows (hq_off)
  void* y;
  int y_f32;
};

constexpr int kWarps = 8;
constexpr float kLimit = 10.0f;  // SwiGLU clamp (dsv41/tt/moe.py:15, 134-135)

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }

// w1|w3 of one 16-row tile for one slot: warps split K; C columns 2u, 2u+1 = (hi, lo) of slot
// token nt * 4 + u.
template <int RFMT, int NTL>
__device__ __forceinline__ void w13_tile(const DecodeArgs& a, int slot, int t, float (*red)[16][32]) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
  const int e = a.slot_expert[slot];
  const bool shared = e >= a.E;
  const int ntok = a.slot_ntok[slot];
  const uint8_t* xr[NTL];
#pragma unroll
  for (int j = 0; j < NTL; ++j) {
    const int tok = a.slot_tok[slot * DSMOE_SLOT_TOKENS + min(4 * j + (g >> 1), ntok - 1)];
    xr[j] = a.xq + ((long long)tok * 2 + (g & 1)) * a.H + tq * 16;
  }
  float acc1[NTL][4], acc3[NTL][4];
#pragma unroll
  for (int j = 0; j < NTL; ++j)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc1[j][q] = acc3[j][q] = 0.f;

  if (RFMT == DSMOE_FMT_FP8 || shared) {
    const uint8_t* tile =
        (shared ? a.s_w13 : a.r_w13 + (long long)e * a.r_w13_eb) + (long long)t * fp8_w13_tile_bytes(a.H);
    const int KB = a.H / 128, KC = a.H / 32;
    const int kb0 = warp * KB / kWarps, kb1 = (warp + 1) * KB / kWarps;
    for (int kb = kb0; kb < kb1; ++kb) {
      uint4 w1v[4], w3v[4], xv[NTL][2];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint8_t* ch = tile + fp8_w13_chunk_off(4 * kb + i) + lane * 16;
        w1v[i] = ld_stream16(ch);
        w3v[i] = ld_stream16(ch + 512);
      }
#pragma unroll
      for (int j = 0; j < NTL; ++j) {
        xv[j][0] = ld16(xr[j] + (2 * kb) * 64);
        xv[j][1] = ld16(xr[j] + (2 * kb + 1) * 64);
      }
      const float* sc = reinterpret_cast<const float*>(tile + fp8_w13_scale_off(kb >> 1, KC));
      const float s1 = __ldg(sc + fp8_w13_scale_index(kb, 0)), s3 = __ldg(sc + fp8_w13_scale_index(kb, 1));
      float u1[NTL][4], u3[NTL][4];
#pragma unroll
      for (int j = 0; j < NTL; ++j)
#pragma unroll
        for (int q = 0; q < 4; ++q) u1[j][q] = u3[j][q] = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
#pragma unroll
        for (int j = 0; j < NTL; ++j) {
          const uint4 xb = xv[j][i >> 1];
          const uint32_t b0 = (i & 1) ? xb.z : xb.x, b1 = (i & 1) ? xb.w : xb.y;
          mma_e4m3(u1[j], w1v[i].x, w1v[i].y, w1v[i].z, w1v[i].w, b0, b1);
          mma_e4m3(u3[j], w3v[i].x, w3v[i].y, w3v[i].z, w3v[i].w, b0, b1);
        }
      }
#pragma unroll
      for (int j = 0; j < NTL; ++j)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          acc1[j][q] = fmaf(u1[j][q], s1, acc1[j][q]);
          acc3[j][q] = fmaf(u3[j][q], s3, acc3[j][q]);
        }
    }
  } else {
    const uint8_t* tile = a.r_w13 + (long long)e * a.r_w13_eb + (long long)t * fp4_w13_tile_bytes(a.H);
    const int KC = a.H / 64;
    const int c0 = warp * KC / kWarps, c1 = (warp + 1) * KC / kWarps;
    for (int c = c0; c < c1; c += 2) {
      const int nch = min(2, c1 - c);
      uint4 w1v[2], w3v[2], xv[2][NTL];
      uint32_t s1v[2], s3v[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        if (i < nch) {
          const uint8_t* ch = tile + (long long)(c + i) * 1088;
          w1v[i] = ld_stream16(ch + lane * 16);
          w3v[i] = ld_stream16(ch + 512 + lane * 16);
          s1v[i] = __ldg(reinterpret_cast<const uint32_t*>(ch + 1024) + g);
          s3v[i] = __ldg(reinterpret_cast<const uint32_t*>(ch + 1056) + g);
#pragma unroll
          for (int j = 0; j < NTL; ++j) xv[i][j] = ld16(xr[j] + (c + i) * 64);
        }
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        if (i < nch) {
          fp4_chunk_mma<NTL>(w1v[i], s1v[i], xv[i], acc1);
          fp4_chunk_mma<NTL>(w3v[i], s3v[i], xv[i], acc3);
        }
      }
    }
  }

#pragma unroll
  for (int j = 0; j < NTL; ++j)
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      red[warp][8 * j + q][lane] = acc1[j][q];
      red[warp][8 * j + 4 + q][lane] = acc3[j][q];
    }
  __syncthreads();
  if (warp < NTL) {  // warp j finishes n-tile j
    const int j = warp;
    float s[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      s[q] = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) s[q] += red[w][8 * j + q][lane];
    }
    const int q = 4 * j + tq;
    if (q < ntok) {
      const int tok = a.slot_tok[slot * DSMOE_SLOT_TOKENS + q];
      const float f = a.xscale[tok] * (RFMT == DSMOE_FMT_FP4 && !shared ? kFp4E4m3Scale : 1.0f);
      float h[2];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const float gv = fminf((s[2 * r] + s[2 * r + 1] * kLoInv) * f, kLimit);
        const float uv = fminf(fmaxf((s[4 + 2 * r] + s[5 + 2 * r] * kLoInv) * f, -kLimit), kLimit);
        h[r] = silu_f(gv) * uv * kHScale;
      }
      uint32_t hi2, lo2;
      split2_e4m3(h[0], h[1], hi2, lo2);
      const int k = 16 * t + g;
      a.hq[hq_off(a.I_loc, slot, q, 0, k)] = (uint8_t)hi2;
      a.hq[hq_off(a.I_loc, slot, q, 0, k + 8)] = (uint8_t)(hi2 >> 8);
      a.hq[hq_off(a.I_loc, slot, q, 1, k)] = (uint8_t)lo2;
      a.hq[hq_off(a.I_loc, slot, q, 1, k + 8)] = (uint8_t)(lo2 >> 8);
    }
  }
}

template <int RFMT>
__global__ void __launch_bounds__(256, 2) moe_w13_kernel(DecodeArgs a) {
  const int slot = blockIdx.y;
  if (slot >= a.plan[0]) return;
  __shared__ float red[kWarps][16][32];  // [warp][n-tile * 8 + matrix * 4 + c][lane]
  if (a.slot_ntok[slot] <= 4)
    w13_tile<RFMT, 1>(a, slot, blockIdx.x, red);
  else
    w13_tile<RFMT, 2>(a, slot, blockIdx.x, red);
}

// A warp's run of n consecutive w2 chunks of one slot, from chunk c, for the CTA's 16 output rows;
// added to the warp's [16][B] tile in token columns with the routing weight.
template <int RFMT, int NTL>
__device__ __forceinline__ void w2_run(const DecodeArgs& a, float* yw, int nt, int slot, int c, int n) {
  const int lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
  const int e = a.slot_expert[slot];
  const bool shared = e >= a.E;
  const int ntok = a.slot_ntok[slot];
  const uint8_t* hr[NTL];
#pragma unroll
  for (int j = 0; j < NTL; ++j)
    hr[j] = a.hq + hq_row(a.I_loc, slot, g & 1, min(4 * j + (g >> 1), ntok - 1)) + tq * 16;
  float acc[NTL][4];
#pragma unroll
  for (int j = 0; j < NTL; ++j)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[j][q] = 0.f;
  if (RFMT == DSMOE_FMT_FP8 || shared) {
    const int KC8 = a.I_loc / 32;
    const uint8_t* tile =
        (shared ? a.s_w2 : a.r_w2 + (long long)e * a.r_w2_eb) + (long long)nt * fp8_w2_tile_bytes(a.I_loc);
    for (int cc = c; cc < c + n; cc += 4) {
      const int m = min(4, c + n - cc);
      uint4 wv[4];
      uint2 hv[4][NTL];
      float s[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (i < m) {
          const int k = cc + i;
          wv[i] = ld_stream16(tile + fp8_w2_chunk_off(k) + lane * 16);
          s[i] = __ldg(reinterpret_cast<const float*>(tile + fp8_w2_scale_off(k >> 3, KC8)) + (k & 7));
#pragma unroll
          for (int j = 0; j < NTL; ++j)
            hv[i][j] = *reinterpret_cast<const uint2*>(hr[j] + (k >> 1) * 64 + (k & 1) * 8);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (i < m) {
#pragma unroll
          for (int j = 0; j < NTL; ++j) {
            float d[4];
            mma_e4m3_z(d, wv[i].x, wv[i].y, wv[i].z, wv[i].w, hv[i][j].x, hv[i][j].y);
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[j][q] = fmaf(d[q], s[i], acc[j][q]);
          }
        }
      }
    }
  } else {
    const uint8_t* tile = a.r_w2 + (long long)e * a.r_w2_eb + (long long)nt * fp4_w2_tile_bytes(a.I_loc);
    constexpr int NB = 1;  // chunks per step (register budget of 2 CTAs per SM)
    for (int cc = c; cc < c + n; cc += NB) {
      const int m = min(NB, c + n - cc);
      uint4 wv[NB], hv[NB][NTL];
      uint32_t sv[NB];
#pragma unroll
      for (int i = 0; i < NB; ++i) {
        if (i < m) {
          const int k = cc + i;
          const uint8_t* ch = tile + (long long)k * 544;
          wv[i] = ld_stream16(ch + lane * 16);
          sv[i] = __ldg(reinterpret_cast<const uint32_t*>(ch + 512) + g);
#pragma unroll
          for (int j = 0; j < NTL; ++j) hv[i][j] = ld16(hr[j] + k * 64);
        }
      }
#pragma unroll
      for (int i = 0; i < NB; ++i)
        if (i < m) fp4_chunk_mma<NTL>(wv[i], sv[i], hv[i], acc);
    }
  }
  const float fs = (RFMT == DSMOE_FMT_FP4 && !shared ? kFp4E4m3Scale : 1.0f) / kHScale;
#pragma unroll
  for (int j = 0; j < NTL; ++j) {
    const int q = 4 * j + tq;
    if (q < ntok) {
      const int tok = a.slot_tok[slot * DSMOE_SLOT_TOKENS + q];
      const float f = a.slot_wt[slot * DSMOE_SLOT_TOKENS + q] * fs;
      yw[g * a.B + tok] += (acc[j][0] + acc[j][1] * kLoInv) * f;
      yw[(g + 8) * a.B + tok] += (acc[j][2] + acc[j][3] * kLoInv) * f;
    }
  }
  __syncwarp();
}

template <int RFMT>
__global__ void __launch_bounds__(256, 2) moe_w2_kernel(DecodeArgs a) {
  extern __shared__ float ysm[];  // [kWarps][16][B]
  const int nt = blockIdx.x;
  const int warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < kWarps * 16 * a.B; i += blockDim.x) ysm[i] = 0.f;
  __syncthreads();
  const int nslots = a.plan[0], nrouted = a.plan[1];
  const int KC8 = a.I_loc / 32;
  const int KCr = RFMT == DSMOE_FMT_FP8 ? KC8 : a.I_loc / 64;
  const long long nr_items = (long long)nrouted * KCr;
  const long long total = nr_items + (long long)(nslots - nrouted) * KC8;
  const long long i0 = warp * total / kWarps, i1 = (warp + 1) * total / kWarps;
  float* yw = ysm + warp * 16 * a.B;

  long long it = i0;
  while (it < i1) {
    int slot, c, nch_slot;
    if (it < nr_items) {
      slot = (int)(it / KCr);
      c = (int)(it % KCr);
      nch_slot = KCr;
    } else {
      const long long r = it - nr_items;
      slot = nrouted + (int)(r / KC8);
      c = (int)(r % KC8);
      nch_slot = KC8;
    }
    const int n = (int)min((long long)(nch_slot - c), i1 - it);
    if (a.slot_ntok[slot] <= 4)
      w2_run<RFMT, 1>(a, yw, nt, slot, c, n);
    else
      w2_run<RFMT, 2>(a, yw, nt, slot, c, n);
    it += n;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 16 * a.B; i += blockDim.x) {
    const int r = i / a.B, tok = i % a.B;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += ysm[(w * 16 + r) * a.B + tok];
    const long long o = (long long)tok * a.H + nt * 16 + r;
    if (a.y_f32)
      reinterpret_cast<float*>(a.y)[o] = s;
    else
      reinterpret_cast<__nv_bfloat16*>(a.y)[o] = __float2bfloat16_rn(s);
  }
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ s, __nv_bfloat16* __restrict__ d, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    d[i] = __float2bfloat16_rn(s[i]);
}

// ------------------------------------------------------------------ workspace and validation
struct WsLayout {
  size_t logits, idx32, wt32, xq, xscale, plan, slot_expert, slot_ntok, slot_tok, slot_wt, hq, total;
};

static size_t al(size_t v) { return (v + 255) & ~size_t(255); }

static WsLayout ws_layout(int B, int H, int E, int topk, int I_loc, size_t base) {
  WsLayout w{};
  const int S = max_slots(B, topk);
  size_t o = base;
  w.logits = o; o += al((size_t)B * E * 4);
  w.idx32 = o; o += al((size_t)B * topk * 4);
  w.wt32 = o; o += al((size_t)B * topk * 4);
  w.xq = o; o += al((size_t)B * 2 * H);
  w.xscale = o; o += al((size_t)B * 4);
  w.plan = o; o += al(16);
  w.slot_expert = o; o += al((size_t)S * 4);
  w.slot_ntok = o; o += al((size_t)S * 4);
  w.slot_tok = o; o += al((size_t)S * DSMOE_SLOT_TOKENS * 4);
  w.slot_wt = o; o += al((size_t)S * DSMOE_SLOT_TOKENS * 4);
  w.hq = o; o += al((size_t)S * hq_slot_bytes(I_loc));
  w.total = o;
  return w;
}

// The persistent path's scratch sits at the front of the workspace, at a size and position that
// depend only on the layer geometry (never on the batch), so calls of any batch share it safely.
static size_t fused_region(const dsmoe_layer_t* L) {
  if (L->inter_local <= 0 || L->inter_local % 32 || L->hidden % 512 ||
      (L->routed.fmt != DSMOE_FMT_FP8 && L->routed.fmt != DSMOE_FMT_FP4))
    return 0;
  return fused_scratch(L->hidden, L->inter_local, L->n_experts, 8, L->topk, L->routed.fmt).total;
}

static bool is_tc(const dsmoe_layer_t* L) { return L->routed.layout == DSMOE_LAYOUT_TC; }

// The multi-kernel path's scratch (dsmoe_router, B > 8) starts after the persistent kernel's, which
// stays at the front: the tensor-core path's (counters included) or the fragment path's.
static WsLayout ws_layout_for(const dsmoe_layer_t* L, int B) {
  const size_t base = is_tc(L) ? tc_scratch(L).total : fused_region(L);
  return ws_layout(B, L->hidden, L->n_experts, L->topk, L->inter_local > 0 ? L->inter_local : 0, base);
}

static int validate(const dsmoe_layer_t* L, int B, bool need_experts) {
  DSMOE_REQUIRE(L, DSMOE_ERR_ARG, "layer is null");
  DSMOE_REQUIRE(B >= 1 && B <= DSMOE_MAX_DECODE_TOKENS, DSMOE_ERR_ARG, "batch %d outside 1..%d", B,
                DSMOE_MAX_DECODE_TOKENS);
  DSMOE_REQUIRE(L->hidden > 0 && L->hidden % 128 == 0, DSMOE_ERR_ARG, "hidden %d must be a multiple of 128", L->hidden);
  DSMOE_REQUIRE(L->n_experts >= 1 && L->n_experts <= 4096, DSMOE_ERR_ARG, "n_experts %d outside 1..4096", L->n_experts);
  DSMOE_REQUIRE(L->topk >= 1 && L->topk <= DSMOE_MAX_TOPK && L->topk <= L->n_experts, DSMOE_ERR_ARG,
                "topk %d outside 1..min(8, n_experts)", L->topk);
  DSMOE_REQUIRE(L->score_func == DSMOE_SCORE_SIGMOID || L->score_func == DSMOE_SCORE_SQRTSOFTPLUS, DSMOE_ERR_ARG,
                "score_func %d", L->score_func);
  DSMOE_REQUIRE(L->gate_w && L->gate_bias, DSMOE_ERR_ARG, "router weights are null");
  DSMOE_REQUIRE(((uintptr_t)L->gate_w & 15) == 0, DSMOE_ERR_ALIGN, "gate_w must be 16-byte aligned");
  if (!need_experts) return DSMOE_OK;
  const dsmoe_store_t& R = L->routed;
  const dsmoe_store_t& S = L->shared;
  DSMOE_REQUIRE(R.fmt == DSMOE_FMT_FP8 || R.fmt == DSMOE_FMT_FP4, DSMOE_ERR_ARG, "routed fmt %d", R.fmt);
  DSMOE_REQUIRE(S.fmt == DSMOE_FMT_FP8 && S.n_experts == 1, DSMOE_ERR_UNSUPPORTED,
                "the shared expert must be one FP8 expert");
  DSMOE_REQUIRE(R.n_experts == L->n_experts, DSMOE_ERR_ARG, "routed store holds %d experts, layer has %d",
                R.n_experts, L->n_experts);
  DSMOE_REQUIRE(R.layout == S.layout && (R.layout == DSMOE_LAYOUT_FRAG || R.layout == DSMOE_LAYOUT_TC),
                DSMOE_ERR_ARG, "store layouts %d / %d", R.layout, S.layout);
  long long e13, e2;
  if (R.layout == DSMOE_LAYOUT_TC) {
    DSMOE_REQUIRE(R.row0 == S.row0, DSMOE_ERR_ARG, "routed and shared slices differ");
    DSMOE_REQUIRE(dsmoe_store_tc_expert_bytes(R.fmt, L->hidden, R.row0 + L->inter_local, R.row0, L->inter_local, &e13,
                                              &e2) == DSMOE_OK, DSMOE_ERR_ARG, "tc store geometry");
    DSMOE_REQUIRE(R.w13_expert_bytes == e13 && R.w2_expert_bytes == e2, DSMOE_ERR_ARG,
                  "routed tc store strides (%lld, %lld) differ from (%lld, %lld)", R.w13_expert_bytes,
                  R.w2_expert_bytes, e13, e2);
    dsmoe_store_tc_expert_bytes(DSMOE_FMT_FP8, L->hidden, R.row0 + L->inter_local, R.row0, L->inter_local, &e13, &e2);
    DSMOE_REQUIRE(S.w13_expert_bytes == e13 && S.w2_expert_bytes == e2, DSMOE_ERR_ARG, "shared tc store strides");
    DSMOE_REQUIRE(R.w13 && R.w2 && S.w13 && S.w2, DSMOE_ERR_ARG, "store pointers are null");
    DSMOE_REQUIRE((((uintptr_t)R.w13 | (uintptr_t)R.w2 | (uintptr_t)S.w13 | (uintptr_t)S.w2) & 1023) == 0,
                  DSMOE_ERR_ALIGN, "tc store pointers must be 1024-byte aligned");
    return DSMOE_OK;
  }
  const int kq = R.fmt == DSMOE_FMT_FP8 ? 32 : 64;
  DSMOE_REQUIRE(L->inter_local > 0 && L->inter_local % kq == 0, DSMOE_ERR_ARG,
                "inter_local %d must be a multiple of %d", L->inter_local, kq);
  dsmoe_store_expert_bytes(R.fmt, L->hidden, L->inter_local, &e13, &e2);
  DSMOE_REQUIRE(R.w13_expert_bytes == e13 && R.w2_expert_bytes == e2, DSMOE_ERR_ARG,
                "routed store strides (%lld, %lld) differ from the packed sizes (%lld, %lld)",
                R.w13_expert_bytes, R.w2_expert_bytes, e13, e2);
  dsmoe_store_expert_bytes(DSMOE_FMT_FP8, L->hidden, L->inter_local, &e13, &e2);
  DSMOE_REQUIRE(S.w13_expert_bytes == e13 && S.w2_expert_bytes == e2, DSMOE_ERR_ARG, "shared store strides");
  DSMOE_REQUIRE(R.w13 && R.w2 && S.w13 && S.w2, DSMOE_ERR_ARG, "store pointers are null");
  DSMOE_REQUIRE((((uintptr_t)R.w13 | (uintptr_t)R.w2 | (uintptr_t)S.w13 | (uintptr_t)S.w2) & 15) == 0,
                DSMOE_ERR_ALIGN, "store pointers must be 16-byte aligned");
  return DSMOE_OK;
}

static RouterArgs router_args(const dsmoe_layer_t* L, const void* x, int B, const uint8_t* image_mask,
                              int64_t* idx, float* wt, float* scores, uint8_t* ws, const WsLayout& w) {
  RouterArgs a{};
  a.x = (const __nv_bfloat16*)x;
  a.B = B;
  a.H = L->hidden;
  a.E = L->n_experts;
  a.topk = L->topk;
  a.score_func = L->score_func;
  a.route_scale = L->route_scale;
  a.wg = L->gate_w;
  a.bias = L->gate_bias;
  a.bias_vl = L->gate_bias_vl;
  a.image_mask = image_mask;
  a.logits = (float*)(ws + w.logits);
  a.idx32 = (int*)(ws + w.idx32);
  a.wt32 = (float*)(ws + w.wt32);
  a.xq = ws + w.xq;
  a.xscale = (float*)(ws + w.xscale);
  a.plan = (int*)(ws + w.plan);
  a.slot_expert = (int*)(ws + w.slot_expert);
  a.slot_ntok = (int*)(ws + w.slot_ntok);
  a.slot_tok = (int*)(ws + w.slot_tok);
  a.slot_wt = (float*)(ws + w.slot_wt);
  a.idx = idx;
  a.wt = wt;
  a.scores = scores;
  return a;
}

}  // namespace dsmoe

using namespace dsmoe;

extern "C" size_t dsmoe_moe_workspace_bytes(const dsmoe_layer_t* L, int B) {
  if (!L || B < 1) return 0;
  return ws_layout_for(L, B).total;
}

extern "C" int dsmoe_router(const dsmoe_layer_t* L, const void* x, int B, const uint8_t* image_mask, int64_t* idx,
                            float* wt, float* scores, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = validate(L, B, false);
  if (rc) return rc;
  DSMOE_REQUIRE(x && workspace, DSMOE_ERR_ARG, "router: x / workspace null");
  DSMOE_REQUIRE(((uintptr_t)x & 7) == 0 && ((uintptr_t)workspace & 255) == 0, DSMOE_ERR_ALIGN,
                "router: x must be 8-byte and workspace 256-byte aligned");
  const WsLayout w = ws_layout_for(L, B);
  DSMOE_REQUIRE(workspace_bytes >= w.total, DSMOE_ERR_WORKSPACE, "router: workspace %zu < %zu", workspace_bytes, w.total);
  RouterArgs a = router_args(L, x, B, image_mask, idx, wt, scores, (uint8_t*)workspace, w);
  return launch_router(a, false, (cudaStream_t)stream);
}

static bool takes_fused(const dsmoe_layer_t* L, const void* x, int B) {
  if (is_tc(L)) return tc_supported(L, B) && ((uintptr_t)x & 15) == 0;
  return fused_region(L) > 0 && fused_supported(L, B) && ((uintptr_t)x & 15) == 0;  // 16-byte token loads
}

static int moe_decode_impl(const dsmoe_layer_t* L, const void* x, int B, const uint8_t* image_mask, void* y,
                           int y_dtype, int64_t* idx, float* wt, float* scores, void* workspace,
                           size_t workspace_bytes, void* stream, void* const* events,
                           const PeerExchange* px = nullptr) {
  int rc = validate(L, B, true);
  if (rc) return rc;
  DSMOE_REQUIRE(x && y && workspace, DSMOE_ERR_ARG, "moe_decode: x / y / workspace null");
  DSMOE_REQUIRE(y_dtype == DSMOE_DTYPE_BF16 || y_dtype == DSMOE_DTYPE_F32, DSMOE_ERR_ARG, "moe_decode: y_dtype %d", y_dtype);
  DSMOE_REQUIRE(((uintptr_t)x & 7) == 0 && ((uintptr_t)workspace & 255) == 0, DSMOE_ERR_ALIGN,
                "moe_decode: x must be 8-byte and workspace 256-byte aligned");
  const WsLayout w = ws_layout_for(L, B);
  DSMOE_REQUIRE(workspace_bytes >= w.total, DSMOE_ERR_WORKSPACE, "moe_decode: workspace %zu < %zu", workspace_bytes,
                w.total);
  uint8_t* ws = (uint8_t*)workspace;
  cudaStream_t st = (cudaStream_t)stream;
  if (is_tc(L)) {
    DSMOE_REQUIRE(workspace_bytes >= tc_scratch(L).total, DSMOE_ERR_WORKSPACE, "moe_decode: workspace %zu < %zu",
                  workspace_bytes, tc_scratch(L).total);
    DSMOE_REQUIRE(takes_fused(L, x, B), DSMOE_ERR_UNSUPPORTED,
                  "moe_decode: the tensor-core store serves batches of 1..8 (x 16-byte aligned); batch %d", B);
    if (events) {
      for (int i = 0; i < 3; ++i) cudaEventRecord((cudaEvent_t)events[i], st);
    }
    rc = launch_tc(L, x, B, image_mask, y, y_dtype, idx, wt, scores, ws, st, px);
    if (events) cudaEventRecord((cudaEvent_t)events[3], st);
    return rc;
  }
  if (takes_fused(L, x, B)) return launch_fused(L, x, B, image_mask, y, y_dtype, idx, wt, scores, ws, st, events, px);
  DSMOE_REQUIRE(!px, DSMOE_ERR_UNSUPPORTED, "moe_decode_allreduce: batch %d / layer shape not on the persistent path", B);
  RouterArgs ra = router_args(L, x, B, image_mask, idx, wt, scores, ws, w);
  if (events) cudaEventRecord((cudaEvent_t)events[0], st);
  rc = launch_router(ra, true, st);
  if (rc) return rc;
  if (events) cudaEventRecord((cudaEvent_t)events[1], st);

  DecodeArgs a{};
  a.H = L->hidden;
  a.I_loc = L->inter_local;
  a.E = L->n_experts;
  a.B = B;
  a.r_fmt = L->routed.fmt;
  a.r_w13 = L->routed.w13;
  a.r_w2 = L->routed.w2;
  a.r_w13_eb = L->routed.w13_expert_bytes;
  a.r_w2_eb = L->routed.w2_expert_bytes;
  a.s_w13 = L->shared.w13;
  a.s_w2 = L->shared.w2;
  a.plan = ra.plan;
  a.slot_expert = ra.slot_expert;
  a.slot_ntok = ra.slot_ntok;
  a.slot_tok = ra.slot_tok;
  a.slot_wt = ra.slot_wt;
  a.xq = ra.xq;
  a.xscale = ra.xscale;
  a.hq = ws + w.hq;
  a.y = y;
  a.y_f32 = y_dtype == DSMOE_DTYPE_F32;
  const dim3 g13(L->inter_local / 16, max_slots(B, L->topk));
  const size_t smem2 = (size_t)kWarps * 16 * B * sizeof(float);
  if (a.r_fmt == DSMOE_FMT_FP8)
    moe_w13_kernel<DSMOE_FMT_FP8><<<g13, 256, 0, st>>>(a);
  else
    moe_w13_kernel<DSMOE_FMT_FP4><<<g13, 256, 0, st>>>(a);
  if (events) cudaEventRecord((cudaEvent_t)events[2], st);
  if (a.r_fmt == DSMOE_FMT_FP8)
    moe_w2_kernel<DSMOE_FMT_FP8><<<L->hidden / 16, 256, smem2, st>>>(a);
  else
    moe_w2_kernel<DSMOE_FMT_FP4><<<L->hidden / 16, 256, smem2, st>>>(a);
  if (events) cudaEventRecord((cudaEvent_t)events[3], st);
  return cuda_status("moe_decode");
}

extern "C" int dsmoe_moe_decode(const dsmoe_layer_t* L, const void* x, int B, const uint8_t* image_mask, void* y,
                                int y_dtype, int64_t* idx, float* wt, float* scores, void* workspace,
                                size_t workspace_bytes, void* stream) {
  return moe_decode_impl(L, x, B, image_mask, y, y_dtype, idx, wt, scores, workspace, workspace_bytes, stream,
                         nullptr);
}

extern "C" int dsmoe_moe_decode_profiled(const dsmoe_layer_t* L, const void* x, int B, const uint8_t* image_mask,
                                         void* y, int y_dtype, int64_t* idx, float* wt, float* scores,
                                         void* workspace, size_t workspace_bytes, void* stream,
                                         void* const* events) {
  DSMOE_REQUIRE(events && events[0] && events[1] && events[2] && events[3], DSMOE_ERR_ARG,
                "moe_decode_profiled: four events required");
  return moe_decode_impl(L, x, B, image_mask, y, y_dtype, idx, wt, scores, workspace, workspace_bytes, stream,
                         events);
}

extern "C" int dsmoe_moe_allreduce_supported(const dsmoe_layer_t* L, const dsmoe_comm_t* comm, const void* x,
                                             int B) {
  const PeerExchange* px = comm_exchange(comm);
  if (!px || !L || !x || validate(L, B, true) != DSMOE_OK || px->hidden != L->hidden) return 0;
  return takes_fused(L, x, B) ? 1 : 0;
}

extern "C" int dsmoe_moe_decode_allreduce(const dsmoe_layer_t* L, const dsmoe_comm_t* comm, const void* x, int B,
                                          const uint8_t* image_mask, void* y, int y_dtype, int64_t* idx, float* wt,
                                          float* scores, void* workspace, size_t workspace_bytes, void* stream) {
  const PeerExchange* px = comm_exchange(comm);
  DSMOE_REQUIRE(px, DSMOE_ERR_ARG, "moe_decode_allreduce: comm is null or not opened");
  return moe_decode_impl(L, x, B, image_mask, y, y_dtype, idx, wt, scores, workspace, workspace_bytes, stream,
                         nullptr, px);
}

extern "C" int dsmoe_moe_check(const dsmoe_layer_t* L, int B, void* workspace, size_t workspace_bytes,
                               void* stream) {
  int rc = validate(L, B, true);
  if (rc) return rc;
  DSMOE_REQUIRE(workspace, DSMOE_ERR_ARG, "moe_check: workspace null");
  cudaStream_t st = (cudaStream_t)stream;
  if (is_tc(L)) {
    const TcScratch f = tc_scratch(L);
    if (workspace_bytes < f.total) return DSMOE_OK;
    if (cudaStreamSynchronize(st) != cudaSuccess) return cuda_status("moe_check: synchronize");
    uint8_t* base = (uint8_t*)workspace;
    unsigned status = 0;
    if (cudaMemcpy(&status, base + f.status, 4, cudaMemcpyDeviceToHost) != cudaSuccess)
      return cuda_status("moe_check: read status");
    if (status == 0) return DSMOE_OK;
    cudaMemsetAsync(base, 0, f.counters_end, st);  // grid counter, status, tagged partials and counters
    cudaStreamSynchronize(st);
    set_error("moe_decode: a bounded device wait expired (status 0x%x); workspace counters were reset", status);
    return DSMOE_ERR_TIMEOUT;
  }
  const WsLayout w = ws_layout_for(L, B);
  if (fused_region(L) == 0 || workspace_bytes < w.total) return DSMOE_OK;
  if (cudaStreamSynchronize(st) != cudaSuccess) return cuda_status("moe_check: synchronize");
  const FusedScratch f = fused_scratch(L->hidden, L->inter_local, L->n_experts, 8, L->topk, L->routed.fmt);
  uint8_t* base = (uint8_t*)workspace;
  unsigned status = 0;
  if (cudaMemcpy(&status, base + f.status, 4, cudaMemcpyDeviceToHost) != cudaSuccess)
    return cuda_status("moe_check: read status");
  if (status == 0) return DSMOE_OK;
  // a bounded wait expired: clear the scratch counters so the next call starts clean
  cudaMemsetAsync(base + f.gbar, 0, f.p13 - f.gbar, st);  // counters, status and tagged router partials
  cudaStreamSynchronize(st);
  set_error("moe_decode: a bounded device wait expired (status 0x%x); workspace counters were reset", status);
  return DSMOE_ERR_TIMEOUT;
}

extern "C" int dsmoe_copy_async(void* dst, const void* src, long long n, void* stream) {
  DSMOE_REQUIRE(dst && src && n >= 0, DSMOE_ERR_ARG, "copy_async: bad arguments");
  if (n == 0) return DSMOE_OK;
  if (cudaMemcpyAsync(dst, src, (size_t)n, cudaMemcpyDefault, (cudaStream_t)stream) != cudaSuccess)
    return cuda_status("copy_async");
  return DSMOE_OK;
}

extern "C" int dsmoe_f32_to_bf16(const float* src, void* dst, long long n, void* stream) {
  DSMOE_REQUIRE(src && dst && n >= 0, DSMOE_ERR_ARG, "f32_to_bf16: bad arguments");
  if (n == 0) return DSMOE_OK;
  const int grid = (int)std::min<long long>((n + 255) / 256, 148 * 8);
  f32_to_bf16_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(src, (__nv_bfloat16*)dst, n);
  return cuda_status("f32_to_bf16");
}
