// On-device router: the reference's Gate, with no host round trip.
//
// The reference runs the fp32 router GEMV on the device, reads the 384 scores back to the host
// every layer, and picks the experts there (dsv41/tt/moe.py:108-129; dsv41/tt/model.py:422). Here
// all of it stays on the GPU:
//   router_logits_kernel  logits[b, e] = x[b] . gate_w[e]   (fp64 accumulation, rounded to fp32)
//   router_select_kernel  score function, bias, top-k, normalized weights; also writes the token
//                         as the two e4m3 terms the expert kernels read (power-of-2 pre-scale)
//   route_plan_kernel     groups the picks by expert into slots of <= 8 tokens (the virtual
//                         buckets of dsv41/tt/moe.py:184-187) plus the shared expert's slots
#include <float.h>

#include "router.cuh"

namespace dsmoe {

// grid (ceil(E / 2), ceil(B / 8)), 256 threads: warp w -> row 2*bx + w/4, K quarter w%4.
__global__ void __launch_bounds__(256) router_logits_kernel(RouterArgs a) {
  __shared__ double part[8][8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 2 + (warp >> 2), q = warp & 3;
  const int tok0 = blockIdx.y * 8;
  const int ntok = min(8, a.B - tok0);
  double acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.0;
  if (row < a.E) {
    const int n4 = a.H / 4;
    const int beg = q * n4 / 4, end = (q + 1) * n4 / 4;
    const float4* w = reinterpret_cast<const float4*>(a.wg + (long long)row * a.H);
    for (int f = beg + lane; f < end; f += 32) {
      const float4 wv = __ldg(w + f);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (j < ntok) {
          const uint2 xv = *reinterpret_cast<const uint2*>(a.x + (long long)(tok0 + j) * a.H + 4 * f);
          const float x0 = __uint_as_float(xv.x << 16), x1 = __uint_as_float(xv.x & 0xFFFF0000u);
          const float x2 = __uint_as_float(xv.y << 16), x3 = __uint_as_float(xv.y & 0xFFFF0000u);
          acc[j] = fma((double)x0, (double)wv.x, acc[j]);
          acc[j] = fma((double)x1, (double)wv.y, acc[j]);
          acc[j] = fma((double)x2, (double)wv.z, acc[j]);
          acc[j] = fma((double)x3, (double)wv.w, acc[j]);
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const double v = warp_sum_d(acc[j]);
    if (lane == 0) part[warp][j] = v;
  }
  __syncthreads();
  if (threadIdx.x < 16) {
    const int r = threadIdx.x >> 3, j = threadIdx.x & 7;
    const int e = blockIdx.x * 2 + r;
    if (e < a.E && j < ntok) {
      const double s = ((part[4 * r][j] + part[4 * r + 1][j]) + part[4 * r + 2][j]) + part[4 * r + 3][j];
      a.logits[(long long)(tok0 + j) * a.E + e] = __double2float_rn(s);
    }
  }
}

__device__ __forceinline__ float score_fn(float l, int func) {
  const double d = (double)l;
  double s;
  if (func == DSMOE_SCORE_SIGMOID) {
    s = 1.0 / (1.0 + exp(-d));
  } else {  // sqrt(softplus), torch's softplus threshold 20
    s = sqrt(d > 20.0 ? d : log1p(exp(d)));
  }
  return __double2float_rn(s);
}

// grid B, 256 threads, dynamic smem 2 * E floats.
__global__ void __launch_bounds__(256) router_select_kernel(RouterArgs a) {
  extern __shared__ float sm[];
  float* sc = sm;
  float* biased = sm + a.E;
  __shared__ float red[8];
  __shared__ int sel[DSMOE_MAX_TOPK];
  const int tok = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const __nv_bfloat16* xr = a.x + (long long)tok * a.H;

  // (a) token -> e4m3 hi / lo rows with a power-of-2 pre-scale: amax * 2^-p in [128, 256)
  float amax = 0.f;
  for (int i = tid; i < a.H; i += blockDim.x) amax = fmaxf(amax, fabsf(__bfloat162float(xr[i])));
  amax = warp_max(amax);
  if (lane == 0) red[warp] = amax;
  __syncthreads();
  if (tid < 32) {
    float m = tid < (int)(blockDim.x >> 5) ? red[tid] : 0.f;
    m = warp_max(m);
    if (tid == 0) red[0] = m;
  }
  __syncthreads();
  amax = red[0];
  int p = 0;
  if (amax > 0.f && amax <= FLT_MAX) {
    int e2;
    frexpf(amax, &e2);  // amax in [2^(e2-1), 2^e2)
    p = e2 - 8;
  }
  const float inv = ldexpf(1.0f, -p);
  if (tid == 0) a.xscale[tok] = ldexpf(1.0f, p);
  uint8_t* xh = a.xq + (long long)tok * 2 * a.H;
  for (int k = 2 * tid; k < a.H; k += 2 * blockDim.x) {
    uint32_t hi2, lo2;
    split2_e4m3(__bfloat162float(xr[k]) * inv, __bfloat162float(xr[k + 1]) * inv, hi2, lo2);
    *reinterpret_cast<uint16_t*>(xh + qk_off(k)) = (uint16_t)hi2;
    *reinterpret_cast<uint16_t*>(xh + a.H + qk_off(k)) = (uint16_t)lo2;
  }

  // (b) scores and selection values
  const bool vl = a.bias_vl != nullptr && a.image_mask != nullptr && a.image_mask[tok] != 0;
  const float* bias = vl ? a.bias_vl : a.bias;
  for (int e = tid; e < a.E; e += blockDim.x) {
    const float s = score_fn(a.logits[(long long)tok * a.E + e], a.score_func);
    sc[e] = s;
    biased[e] = s + bias[e];
    if (a.scores) a.scores[(long long)tok * a.E + e] = s;
  }
  __syncthreads();

  // (c) top-k by repeated warp argmax; ties go to the lower expert index
  if (warp == 0) {
    for (int r = 0; r < a.topk; ++r) {
      float best = -INFINITY;
      int bi = 0x7FFFFFFF;
      for (int e = lane; e < a.E; e += 32) {
        const float v = biased[e];
        if (v > best || (v == best && e < bi)) { best = v; bi = e; }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
      }
      if (lane == 0) {
        if (bi == 0x7FFFFFFF) bi = 0;  // all -inf / NaN: fall back to expert 0 deterministically
        sel[r] = bi;
        biased[bi] = -INFINITY;
      }
      __syncwarp();
    }
    if (lane == 0) {
      float tot = 0.f;
      for (int r = 0; r < a.topk; ++r) tot += sc[sel[r]];
      for (int r = 0; r < a.topk; ++r) {
        const float w = sc[sel[r]] / (tot + 1e-20f) * a.route_scale;
        const long long o = (long long)tok * a.topk + r;
        a.idx32[o] = sel[r];
        a.wt32[o] = w;
        if (a.idx) a.idx[o] = sel[r];
        if (a.wt) a.wt[o] = w;
      }
    }
  }
}

// One CTA: slot plan for the step. Deterministic: slots ordered by expert id, tokens ascending.
__global__ void __launch_bounds__(512) route_plan_kernel(RouterArgs a) {
  extern __shared__ unsigned long long mask[];  // [E]
  __shared__ int wsum[16];
  const int tid = threadIdx.x, nthr = blockDim.x;
  for (int e = tid; e < a.E; e += nthr) mask[e] = 0ull;
  __syncthreads();
  for (int i = tid; i < a.B * a.topk; i += nthr) atomicOr(&mask[a.idx32[i]], 1ull << (i / a.topk));
  __syncthreads();
  // exclusive scan of slots-per-expert: each thread owns a contiguous run of experts
  const int per = (a.E + nthr - 1) / nthr;
  const int e0 = tid * per, e1 = min(a.E, e0 + per);
  int mine = 0;
  for (int e = e0; e < e1; ++e) mine += (__popcll(mask[e]) + DSMOE_SLOT_TOKENS - 1) / DSMOE_SLOT_TOKENS;
  const int lane = tid & 31, warp = tid >> 5;
  int incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  int woff = 0;
  for (int w = 0; w < warp; ++w) woff += wsum[w];
  int base = woff + incl - mine;
  for (int e = e0; e < e1; ++e) {
    unsigned long long m = mask[e];
    int i = 0;
    const int cnt = __popcll(m);
    while (m) {
      const int tok = __ffsll((long long)m) - 1;
      m &= m - 1;
      const int s = base + i / DSMOE_SLOT_TOKENS, pos = i % DSMOE_SLOT_TOKENS;
      float w = 0.f;
      for (int kk = 0; kk < a.topk; ++kk)
        if (a.idx32[tok * a.topk + kk] == e) w = a.wt32[tok * a.topk + kk];
      a.slot_tok[s * DSMOE_SLOT_TOKENS + pos] = tok;
      a.slot_wt[s * DSMOE_SLOT_TOKENS + pos] = w;
      if (pos == 0) {
        a.slot_expert[s] = e;
        a.slot_ntok[s] = min(DSMOE_SLOT_TOKENS, cnt - i);
      }
      ++i;
    }
    base += (cnt + DSMOE_SLOT_TOKENS - 1) / DSMOE_SLOT_TOKENS;
  }
  __syncthreads();
  if (tid == nthr - 1) {
    const int n_routed = base;  // the last thread's running base is the routed total
    const int n_shared = (a.B + DSMOE_SLOT_TOKENS - 1) / DSMOE_SLOT_TOKENS;
    for (int q = 0; q < n_shared; ++q) {
      const int s = n_routed + q;
      a.slot_expert[s] = a.E;  // the shared expert
      a.slot_ntok[s] = min(DSMOE_SLOT_TOKENS, a.B - q * DSMOE_SLOT_TOKENS);
      for (int pos = 0; pos < DSMOE_SLOT_TOKENS; ++pos) {
        a.slot_tok[s * DSMOE_SLOT_TOKENS + pos] = min(q * DSMOE_SLOT_TOKENS + pos, a.B - 1);
        a.slot_wt[s * DSMOE_SLOT_TOKENS + pos] = 1.0f;
      }
    }
    a.plan[0] = n_routed + n_shared;
    a.plan[1] = n_routed;
  }
}

int launch_router(const RouterArgs& a, bool with_plan, cudaStream_t st) {
  dim3 g1((a.E + 1) / 2, (a.B + 7) / 8);
  router_logits_kernel<<<g1, 256, 0, st>>>(a);
  router_select_kernel<<<a.B, 256, 2 * a.E * sizeof(float), st>>>(a);
  if (with_plan) route_plan_kernel<<<1, 512, a.E * sizeof(unsigned long long), st>>>(a);
  return cuda_status("router");
}

}  // namespace dsmoe
