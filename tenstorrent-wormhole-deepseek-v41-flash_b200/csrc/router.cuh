// Router / slot-plan interface shared by router.cu and moe_decode.cu.
#pragma once
#include "common.cuh"

#define DSMOE_MAX_TOPK 8

namespace dsmoe {

struct RouterArgs {
  const __nv_bfloat16* x;  // [B, H]
  int B, H, E, topk, score_func;
  float route_scale;
  const float* wg;         // [E, H]
  const float* bias;       // [E]
  const float* bias_vl;    // [E] or null
  const uint8_t* image_mask;  // [B] or null
  // workspace
  float* logits;           // [B, E]
  int* idx32;              // [B, k]
  float* wt32;             // [B, k]
  uint8_t* xq;             // [B][2 terms][H] e4m3 hi / lo rows in B-operand order (qk_off)
  float* xscale;           // [B] power of 2 undoing the pre-scale of xq
  int* plan;               // [0] = slots, [1] = routed slots
  int* slot_expert;        // [MAXS] expert id, E = the shared expert
  int* slot_ntok;          // [MAXS]
  int* slot_tok;           // [MAXS][8]
  float* slot_wt;          // [MAXS][8]
  // optional outputs
  int64_t* idx;            // [B, k]
  float* wt;               // [B, k]
  float* scores;           // [B, E]
};

// SwiGLU output h of one slot for w2, the B operand of its 8-bit MMAs: rows of hq_row_bytes, hi
// rows of the 8 slot tokens then lo rows of the 8 slot tokens, K within a row in qk_off order. h
// is stored times kHScale (|SiLU(min(g, 10)) * clamp(u, +-10)| <= 100, so 400 stays inside e4m3's
// 448); the routing weight and 1/kHScale are applied to w2's fp32 output.
constexpr float kHScale = 4.0f;
__host__ __device__ inline int hq_row_bytes(int I_loc) { return (I_loc + 63) / 64 * 64; }
__host__ __device__ inline long long hq_slot_bytes(int I_loc) {
  return 2LL * DSMOE_SLOT_TOKENS * hq_row_bytes(I_loc);
}
__host__ __device__ inline long long hq_row(int I_loc, int slot, int term, int q) {
  return slot * hq_slot_bytes(I_loc) + (long long)(term * DSMOE_SLOT_TOKENS + q) * hq_row_bytes(I_loc);
}
__host__ __device__ inline long long hq_off(int I_loc, int slot, int q, int term, int k) {
  return hq_row(I_loc, slot, term, q) + qk_off(k);
}

// Upper bound on slots in one step: every pick its own slot, plus the shared expert's.
inline int max_slots(int B, int topk) {
  return B * topk + (B + DSMOE_SLOT_TOKENS - 1) / DSMOE_SLOT_TOKENS;
}

int launch_router(const RouterArgs& a, bool with_plan, cudaStream_t st);

// Workspace scratch of the persistent decode kernel (moe_fused.cu); counters first.
struct FusedScratch {
  size_t rl, p13, p2, hq, cnt13, cnt2, slot_done, gbar, status, total;
  int p13max, p2max, slots;
};
FusedScratch fused_scratch(int H, int I_loc, int E, int B, int topk, int r_fmt);
bool fused_supported(const dsmoe_layer_t* L, int B);

// Scratch of the tensor-core decode path (moe_tc.cu) in the caller's workspace; the grid counter
// and the status word sit at the same offsets as in FusedScratch.
struct TcScratch {
  size_t gbar, status, rl, cnt, counters_end, p13, p2, hb, total;
  int slot_cap, cnt_words;
};
TcScratch tc_scratch(const dsmoe_layer_t* L);
bool tc_supported(const dsmoe_layer_t* L, int B);

// Peer exchange of the persistent kernel's all-reduce (comm.cu owns the memory). Every rank has one
// exchange buffer: a control word (the epoch of its last call) and the slots its peers write,
// [2 parities][world source ranks][hidden / 16 output tiles][32 lanes][4 words]; slots[q] is rank
// q's buffer as this GPU addresses it (its own for q == rank, an IPC mapping otherwise).
constexpr int kMaxWorld = 8;
struct PeerExchange {
  int rank, world, hidden;
  unsigned* ctl;
  unsigned long long* slots[kMaxWorld];
};
inline size_t exchange_slot_words(int world, int hidden) { return 2ull * world * (hidden / 16) * 128; }
// The exchange of an opened comm (comm.cu), or nullptr.
const PeerExchange* comm_exchange(const dsmoe_comm_t* c);
int launch_tc(const dsmoe_layer_t* L, const void* x, int B, const uint8_t* image_mask, void* y, int y_dtype,
              int64_t* idx, float* wt, float* scores, uint8_t* ws, cudaStream_t st, const PeerExchange* px);

int launch_fused(const dsmoe_layer_t* L, const void* x, int B, const uint8_t* image_mask, void* y, int y_dtype,
                 int64_t* idx, float* wt, float* scores, uint8_t* ws, cudaStream_t st, void* const* events,
                 const PeerExchange* px = nullptr);

}  // namespace dsmoe
