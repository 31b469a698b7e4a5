// One-shot all-reduce of 16-row output tiles over the tensor-parallel ranks, on NVLink peer memory
// (CUDA IPC mappings of every rank's exchange buffer, comm.cu). Used inside the persistent decode
// kernel (moe_fused.cu) and by the stand-alone row all-reduce (comm.cu).
//
// A tile is 32 lanes x 4 fp32 (lane l: rows l/4 and l/4 + 8 of the tile, tokens 2 (l%4) and
// 2 (l%4) + 1). Each rank stores its partial into slot (parity, its rank, tile) of every peer's
// buffer, then reads the peers' partials of the tile from its own buffer and sums all ranks'
// partials in rank order, so every rank computes the same bits.
// Words are LL pairs: the value's bits in the low half and the call's epoch in the high half. An
// aligned 8-byte store is single-copy atomic, so a reader that sees this call's epoch in a word
// sees the value written with it; no fence or flag is needed. Epochs grow by one per call (the
// control word of the buffer), and slots alternate between two parities: a peer can be at most one
// call ahead (it cannot finish call e + 1 without this rank's tiles of call e + 1), so it never
// overwrites a slot this rank still reads.
#pragma once
#include "router.cuh"

namespace dsmoe {

__device__ __forceinline__ unsigned long long ll_word(float v, unsigned ep) {
  return ((unsigned long long)ep << 32) | __float_as_uint(v);
}
__device__ __forceinline__ void st_ll2(unsigned long long* p, unsigned long long w0, unsigned long long w1) {
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(w0), "l"(w1) : "memory");
}
__device__ __forceinline__ void ld_ll2(const unsigned long long* p, unsigned long long& w0, unsigned long long& w1) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(w0), "=l"(w1) : "l"(p) : "memory");
}
__device__ __forceinline__ size_t ar_slot(int par, int q, int W, int NT, int nt, int lane) {
  return ((((size_t)par * W + q) * NT + nt) * 32 + lane) * 4;
}

// The whole warp calls it for tile nt of NT with the call's B tokens; s4 in: this rank's partial,
// out: the rank-order sum. Only lanes holding a token column below B (2 (lane % 4) < B) send and
// wait; with one token a lane's payload is .x and .z (token 0 of rows lane / 4 and lane / 4 + 8), one
// 16-byte word pair per peer. Per peer a tile therefore costs 128 B at B = 1, 256 B at B = 2, 512 B
// at B <= 4 and 1 KB above. Waits at most limit_ns for the peers; false (for every lane) if a peer's
// words did not arrive.
__device__ __forceinline__ bool ll_allreduce_tile(unsigned long long* const* slots, int W, int r, int NT, int nt,
                                                  int B, unsigned ep, float4& s4, int lane, uint64_t limit_ns) {
  bool ok = true;
  if (2 * (lane & 3) < B) {
    const bool one = B == 1;
    const int par = (int)(ep & 1u);
    const unsigned long long w0 = ll_word(s4.x, ep), w1 = ll_word(one ? s4.z : s4.y, ep), w2 = ll_word(s4.z, ep),
                             w3 = ll_word(s4.w, ep);
    const size_t mine = ar_slot(par, r, W, NT, nt, lane);
    for (int d = 1; d < W; ++d) {  // peers in the order r+1, r+2, ... (spreads the first stores)
      const int q = r + d < W ? r + d : r + d - W;
      unsigned long long* p = slots[q] + mine;
      st_ll2(p, w0, w1);
      if (!one) st_ll2(p + 2, w2, w3);
    }
    // every peer's slot polled together: one round of loads per poll, not one per peer
    float4 v[kMaxWorld];
    unsigned got = 1u << r;  // ranks whose words have arrived
    v[r] = one ? make_float4(s4.x, 0.f, s4.z, 0.f) : s4;
    const unsigned all = (1u << W) - 1u;
    const uint64_t t0 = globaltimer_ns();
    while (got != all) {
      unsigned long long x[kMaxWorld][4];
#pragma unroll
      for (int q = 0; q < kMaxWorld; ++q)
        if (q < W && !((got >> q) & 1u)) {
          const unsigned long long* p = slots[r] + ar_slot(par, q, W, NT, nt, lane);
          ld_ll2(p, x[q][0], x[q][1]);
          if (one) {
            x[q][2] = x[q][1];
            x[q][3] = x[q][0] & 0xFFFFFFFF00000000ull;  // epoch, value 0
          } else {
            ld_ll2(p + 2, x[q][2], x[q][3]);
          }
        }
#pragma unroll
      for (int q = 0; q < kMaxWorld; ++q)
        if (q < W && !((got >> q) & 1u) && (unsigned)(x[q][0] >> 32) == ep && (unsigned)(x[q][1] >> 32) == ep &&
            (unsigned)(x[q][2] >> 32) == ep && (unsigned)(x[q][3] >> 32) == ep) {
          // one token: words (x, z) -> (x, 0, z, 0)
          v[q] = one ? make_float4(__uint_as_float((unsigned)x[q][0]), 0.f, __uint_as_float((unsigned)x[q][1]), 0.f)
                     : make_float4(__uint_as_float((unsigned)x[q][0]), __uint_as_float((unsigned)x[q][1]),
                                   __uint_as_float((unsigned)x[q][2]), __uint_as_float((unsigned)x[q][3]));
          got |= 1u << q;
        }
      if (got != all && globaltimer_ns() - t0 > limit_ns) {
        ok = false;
        break;
      }
    }
    float4 tot = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q = 0; q < W; ++q) {  // rank order: the same bits on every rank
      const float4 u = ((got >> q) & 1u) ? v[q] : make_float4(0.f, 0.f, 0.f, 0.f);
      tot.x += u.x;
      tot.y += u.y;
      tot.z += u.z;
      tot.w += u.w;
    }
    s4 = tot;
  }
  return __all_sync(0xffffffffu, ok);
}

}  // namespace dsmoe
