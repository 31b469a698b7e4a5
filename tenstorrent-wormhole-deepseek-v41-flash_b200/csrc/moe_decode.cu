// Decode-regime MoE layer (1..64 tokens): fused dequant + tensor-core GEMV over resident experts.
//
// Reference path replaced: MoE.decode (dsv41/tt/moe.py:148-180) -- slot gather of the six host-
// chosen experts into concatenated buffers (dsv41/kernels/slot_cat.cpp:194-365), three matmuls,
// the Q20 SwiGLU kernel (dsv41/kernels/slot_cat.cpp:82-192) and the weighted combine -- and its
// multi-token form verify_batched (dsv41/tt/moe.py:202-241).
//
// Per step (after the router kernels, router.cu):
//   moe_w13_kernel  grid (inter_local/16 tiles, slots): one CTA streams one 16-row tile of w1 and
//                   of w3 for one slot (expert + up to 8 tokens), 8 warps split K, mma.sync f16
//                   with fp32 accumulation, per-block (FP8) or per-32 (FP4) scales applied to the
//                   fp32 partials; epilogue: clamp, SiLU(g)*u, routing weight, write h (f16) in the
//                   fragment order w2 reads.
//   moe_w2_kernel   grid hidden/16: one CTA owns 16 output rows for all slots and all tokens;
//                   warps split the (slot, K-chunk) items evenly; deterministic combine in smem.
// Both kernels are HBM-bound: every weight byte of the touched experts is read exactly once per
// step, with 16-byte streaming loads, 4 independent chunks in flight per warp.
#include "router.cuh"

namespace dsmoe {

// fused persistent path (moe_fused.cu)
struct FusedScratch {
  size_t rl, p13, p2, hf, cnt13, cnt2, gbar, status, total;
  int p13max, qmax, slots;
};
FusedScratch fused_scratch(int H, int I_loc, int E, int B, int topk, int r_fmt);
bool fused_supported(const dsmoe_layer_t* L, int B);
int launch_fused(const dsmoe_layer_t* L, const void* x, int B, const uint8_t* image_mask, void* y, int y_dtype,
                 int64_t* idx, float* wt, float* scores, uint8_t* ws, cudaStream_t st, void* const* events);

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
  const uint32_t* xf;
  const float* xscale;
  uint16_t* hf;  // [slots * 8 rows][I_loc] f16, fragment order
  void* y;
  int y_f32;
};

constexpr int kWarps = 8;
constexpr float kLimit = 10.0f;  // SwiGLU clamp (dsv41/tt/moe.py:15, 134-135)

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }

// position of intermediate row j inside a fragment-ordered f16 row (see router.cu, xf layout)
__device__ __forceinline__ int frag_pos(int j) {
  const int k = j & 31, s = k >> 4, kk = k & 15;
  return (j >> 5) * 32 + ((kk & 7) >> 1) * 8 + (2 * s + (kk >> 3)) * 2 + (kk & 1);
}

__device__ __forceinline__ void fma4(float (&acc)[4], const float (&t)[4], float s) {
#pragma unroll
  for (int j = 0; j < 4; ++j) acc[j] = fmaf(t[j], s, acc[j]);
}
// FP4: rows g (c0, c1) and g+8 (c2, c3) carry their own scales
__device__ __forceinline__ void fma4_rows(float (&acc)[4], const float (&t)[4], float s_lo, float s_hi) {
  acc[0] = fmaf(t[0], s_lo, acc[0]);
  acc[1] = fmaf(t[1], s_lo, acc[1]);
  acc[2] = fmaf(t[2], s_hi, acc[2]);
  acc[3] = fmaf(t[3], s_hi, acc[3]);
}

template <int RFMT>
__global__ void __launch_bounds__(256, 2) moe_w13_kernel(DecodeArgs a) {
  const int slot = blockIdx.y;
  if (slot >= a.plan[0]) return;
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
  const int e = a.slot_expert[slot];
  const bool shared = e >= a.E;
  const int ntok = a.slot_ntok[slot];
  const int mytok = a.slot_tok[slot * DSMOE_SLOT_TOKENS + min(g, ntok - 1)];
  const uint4* xrow = reinterpret_cast<const uint4*>(a.xf) + (long long)mytok * (a.H / 32) * 4 + tq;

  float acc1[4] = {0.f, 0.f, 0.f, 0.f}, acc3[4] = {0.f, 0.f, 0.f, 0.f};
  if (RFMT == DSMOE_FMT_FP8 || shared) {
    const uint8_t* tile =
        (shared ? a.s_w13 : a.r_w13 + (long long)e * a.r_w13_eb) + (long long)t * fp8_w13_tile_bytes(a.H);
    const int KB = a.H / 128, KC = a.H / 32;
    const int kb0 = warp * KB / kWarps, kb1 = (warp + 1) * KB / kWarps;
    for (int kb = kb0; kb < kb1; ++kb) {
      uint4 w1v[4], w3v[4], xv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint8_t* ch = tile + fp8_w13_chunk_off(4 * kb + i) + lane * 16;
        w1v[i] = ld_stream16(ch);
        w3v[i] = ld_stream16(ch + 512);
        xv[i] = xrow[(4 * kb + i) * 4];
      }
      const float* sc = reinterpret_cast<const float*>(tile + fp8_w13_scale_off(kb >> 1, KC));
      const float s1 = __ldg(sc + fp8_w13_scale_index(kb, 0)), s3 = __ldg(sc + fp8_w13_scale_index(kb, 1));
      float t1[4] = {0.f, 0.f, 0.f, 0.f}, t3[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint32_t A[4];
        a_frag_fp8(A, w1v[i].x, w1v[i].y);
        mma16816(t1, A, xv[i].x, xv[i].y);
        a_frag_fp8(A, w3v[i].x, w3v[i].y);
        mma16816(t3, A, xv[i].x, xv[i].y);
        a_frag_fp8(A, w1v[i].z, w1v[i].w);
        mma16816(t1, A, xv[i].z, xv[i].w);
        a_frag_fp8(A, w3v[i].z, w3v[i].w);
        mma16816(t3, A, xv[i].z, xv[i].w);
      }
      fma4(acc1, t1, s1);
      fma4(acc3, t3, s3);
    }
  } else {
    const uint8_t* tile = a.r_w13 + (long long)e * a.r_w13_eb + (long long)t * fp4_w13_tile_bytes(a.H);
    const int KC = a.H / 64;
    const int c0 = warp * KC / kWarps, c1 = (warp + 1) * KC / kWarps;
    for (int c = c0; c < c1; c += 2) {
      const int nch = min(2, c1 - c);
      uint4 w1v[2], w3v[2], xv[4];
      uint32_t s1v[2], s3v[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        if (i < nch) {
          const uint8_t* ch = tile + (long long)(c + i) * 1088;
          w1v[i] = ld_stream16(ch + lane * 16);
          w3v[i] = ld_stream16(ch + 512 + lane * 16);
          s1v[i] = __ldg(reinterpret_cast<const uint32_t*>(ch + 1024) + g);
          s3v[i] = __ldg(reinterpret_cast<const uint32_t*>(ch + 1056) + g);
          xv[2 * i] = xrow[(2 * (c + i)) * 4];
          xv[2 * i + 1] = xrow[(2 * (c + i) + 1) * 4];
        }
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        if (i < nch) {
#pragma unroll
          for (int grp = 0; grp < 2; ++grp) {
            const uint4 xb = xv[2 * i + grp];
            const uint32_t wa1 = grp ? w1v[i].z : w1v[i].x, wb1 = grp ? w1v[i].w : w1v[i].y;
            const uint32_t wa3 = grp ? w3v[i].z : w3v[i].x, wb3 = grp ? w3v[i].w : w3v[i].y;
            float t1[4] = {0.f, 0.f, 0.f, 0.f}, t3[4] = {0.f, 0.f, 0.f, 0.f};
            uint32_t A[4];
            a_frag_fp4(A, wa1);
            mma16816(t1, A, xb.x, xb.y);
            a_frag_fp4(A, wb1);
            mma16816(t1, A, xb.z, xb.w);
            a_frag_fp4(A, wa3);
            mma16816(t3, A, xb.x, xb.y);
            a_frag_fp4(A, wb3);
            mma16816(t3, A, xb.z, xb.w);
            fma4_rows(acc1, t1, e8m0_to_f32(s1v[i] >> (8 * grp)), e8m0_to_f32(s1v[i] >> (8 * grp + 16)));
            fma4_rows(acc3, t3, e8m0_to_f32(s3v[i] >> (8 * grp)), e8m0_to_f32(s3v[i] >> (8 * grp + 16)));
          }
        }
      }
    }
  }

  __shared__ float red[kWarps][8][32];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    red[warp][j][lane] = acc1[j];
    red[warp][4 + j][lane] = acc3[j];
  }
  __syncthreads();
  if (warp == 0) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float gs = 0.f, us = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        gs += red[w][q][lane];
        us += red[w][4 + q][lane];
      }
      const int row = q >= 2 ? g + 8 : g, col = 2 * tq + (q & 1);
      if (col < ntok) {
        const int tok = a.slot_tok[slot * DSMOE_SLOT_TOKENS + col];
        const float xs = a.xscale[tok];
        const float gv = fminf(gs * xs, kLimit);
        const float uv = fminf(fmaxf(us * xs, -kLimit), kLimit);
        const float h = silu_f(gv) * uv * a.slot_wt[slot * DSMOE_SLOT_TOKENS + col];
        const int j = 16 * t + row;
        a.hf[(long long)(slot * DSMOE_SLOT_TOKENS + col) * a.I_loc + frag_pos(j)] =
            __half_as_ushort(__float2half_rn(h));
      }
    }
  }
}

// Per-warp accumulation of one slot's 16 x 8 partial into the CTA's [16][B] tile of this warp.
__device__ __forceinline__ void flush_slot(const DecodeArgs& a, float* yw, int slot, const float (&acc)[4],
                                           int g, int tq) {
  const int ntok = a.slot_ntok[slot];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int row = q >= 2 ? g + 8 : g, col = 2 * tq + (q & 1);
    if (col < ntok) yw[row * a.B + a.slot_tok[slot * DSMOE_SLOT_TOKENS + col]] += acc[q];
  }
  __syncwarp();
}

template <int RFMT>
__global__ void __launch_bounds__(256, 2) moe_w2_kernel(DecodeArgs a) {
  extern __shared__ float ysm[];  // [kWarps][16][B]
  const int nt = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
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
    const int e = a.slot_expert[slot];
    const bool shared = e >= a.E;
    const uint4* hrow =
        reinterpret_cast<const uint4*>(a.hf + (long long)(slot * DSMOE_SLOT_TOKENS + g) * a.I_loc) + tq;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    if (RFMT == DSMOE_FMT_FP8 || shared) {
      const uint8_t* tile =
          (shared ? a.s_w2 : a.r_w2 + (long long)e * a.r_w2_eb) + (long long)nt * fp8_w2_tile_bytes(a.I_loc);
      for (int cc = c; cc < c + n; cc += 4) {
        const int m = min(4, c + n - cc);
        uint4 wv[4], hv[4];
        float s[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (i < m) {
            wv[i] = ld_stream16(tile + fp8_w2_chunk_off(cc + i) + lane * 16);
            hv[i] = hrow[(cc + i) * 4];
            s[i] = __ldg(reinterpret_cast<const float*>(tile + fp8_w2_scale_off((cc + i) >> 3, KC8)) + ((cc + i) & 7));
          }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (i < m) {
            float tt[4] = {0.f, 0.f, 0.f, 0.f};
            uint32_t A[4];
            a_frag_fp8(A, wv[i].x, wv[i].y);
            mma16816(tt, A, hv[i].x, hv[i].y);
            a_frag_fp8(A, wv[i].z, wv[i].w);
            mma16816(tt, A, hv[i].z, hv[i].w);
            fma4(acc, tt, s[i]);
          }
        }
      }
    } else {
      const uint8_t* tile = a.r_w2 + (long long)e * a.r_w2_eb + (long long)nt * fp4_w2_tile_bytes(a.I_loc);
      for (int cc = c; cc < c + n; cc += 2) {
        const int m = min(2, c + n - cc);
        uint4 wv[2], hv[4];
        uint32_t sv[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          if (i < m) {
            const uint8_t* ch = tile + (long long)(cc + i) * 544;
            wv[i] = ld_stream16(ch + lane * 16);
            sv[i] = __ldg(reinterpret_cast<const uint32_t*>(ch + 512) + g);
            hv[2 * i] = hrow[(2 * (cc + i)) * 4];
            hv[2 * i + 1] = hrow[(2 * (cc + i) + 1) * 4];
          }
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          if (i < m) {
#pragma unroll
            for (int grp = 0; grp < 2; ++grp) {
              const uint4 hb = hv[2 * i + grp];
              float tt[4] = {0.f, 0.f, 0.f, 0.f};
              uint32_t A[4];
              a_frag_fp4(A, grp ? wv[i].z : wv[i].x);
              mma16816(tt, A, hb.x, hb.y);
              a_frag_fp4(A, grp ? wv[i].w : wv[i].y);
              mma16816(tt, A, hb.z, hb.w);
              fma4_rows(acc, tt, e8m0_to_f32(sv[i] >> (8 * grp)), e8m0_to_f32(sv[i] >> (8 * grp + 16)));
            }
          }
        }
      }
    }
    flush_slot(a, yw, slot, acc, g, tq);
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
  size_t logits, idx32, wt32, xf, xscale, plan, slot_expert, slot_ntok, slot_tok, slot_wt, hf, total;
};

static size_t al(size_t v) { return (v + 255) & ~size_t(255); }

static WsLayout ws_layout(int B, int H, int E, int topk, int I_loc, size_t base) {
  WsLayout w{};
  const int S = max_slots(B, topk);
  size_t o = base;
  w.logits = o; o += al((size_t)B * E * 4);
  w.idx32 = o; o += al((size_t)B * topk * 4);
  w.wt32 = o; o += al((size_t)B * topk * 4);
  w.xf = o; o += al((size_t)B * H * 2);
  w.xscale = o; o += al((size_t)B * 4);
  w.plan = o; o += al(16);
  w.slot_expert = o; o += al((size_t)S * 4);
  w.slot_ntok = o; o += al((size_t)S * 4);
  w.slot_tok = o; o += al((size_t)S * DSMOE_SLOT_TOKENS * 4);
  w.slot_wt = o; o += al((size_t)S * DSMOE_SLOT_TOKENS * 4);
  w.hf = o; o += al((size_t)S * DSMOE_SLOT_TOKENS * I_loc * 2);
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

static WsLayout ws_layout_for(const dsmoe_layer_t* L, int B) {
  return ws_layout(B, L->hidden, L->n_experts, L->topk, L->inter_local > 0 ? L->inter_local : 0, fused_region(L));
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
  const int kq = R.fmt == DSMOE_FMT_FP8 ? 32 : 64;
  DSMOE_REQUIRE(L->inter_local > 0 && L->inter_local % kq == 0, DSMOE_ERR_ARG,
                "inter_local %d must be a multiple of %d", L->inter_local, kq);
  long long e13, e2;
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
  a.xf = (uint32_t*)(ws + w.xf);
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

static int moe_decode_impl(const dsmoe_layer_t* L, const void* x, int B, const uint8_t* image_mask, void* y,
                           int y_dtype, int64_t* idx, float* wt, float* scores, void* workspace,
                           size_t workspace_bytes, void* stream, void* const* events) {
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
  if (fused_region(L) > 0 && fused_supported(L, B))
    return launch_fused(L, x, B, image_mask, y, y_dtype, idx, wt, scores, ws, st, events);
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
  a.xf = ra.xf;
  a.xscale = ra.xscale;
  a.hf = (uint16_t*)(ws + w.hf);
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

extern "C" int dsmoe_moe_check(const dsmoe_layer_t* L, int B, void* workspace, size_t workspace_bytes,
                               void* stream) {
  int rc = validate(L, B, true);
  if (rc) return rc;
  DSMOE_REQUIRE(workspace, DSMOE_ERR_ARG, "moe_check: workspace null");
  const WsLayout w = ws_layout_for(L, B);
  if (fused_region(L) == 0 || workspace_bytes < w.total) return DSMOE_OK;
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaStreamSynchronize(st) != cudaSuccess) return cuda_status("moe_check: synchronize");
  const FusedScratch f = fused_scratch(L->hidden, L->inter_local, L->n_experts, 8, L->topk, L->routed.fmt);
  uint8_t* base = (uint8_t*)workspace;
  unsigned status = 0;
  if (cudaMemcpy(&status, base + f.status, 4, cudaMemcpyDeviceToHost) != cudaSuccess)
    return cuda_status("moe_check: read status");
  if (status == 0) return DSMOE_OK;
  // a bounded wait expired: clear the scratch counters so the next call starts clean
  cudaMemsetAsync(base + f.gbar, 0, f.rl - f.gbar, st);
  cudaStreamSynchronize(st);
  set_error("moe_decode: a bounded device wait expired (status 0x%x); workspace counters were reset", status);
  return DSMOE_ERR_TIMEOUT;
}

extern "C" int dsmoe_f32_to_bf16(const float* src, void* dst, long long n, void* stream) {
  DSMOE_REQUIRE(src && dst && n >= 0, DSMOE_ERR_ARG, "f32_to_bf16: bad arguments");
  if (n == 0) return DSMOE_OK;
  const int grid = (int)std::min<long long>((n + 255) / 256, 148 * 8);
  f32_to_bf16_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(src, (__nv_bfloat16*)dst, n);
  return cuda_status("f32_to_bf16");
}
