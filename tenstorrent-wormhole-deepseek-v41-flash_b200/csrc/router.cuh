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
  uint32_t* xf;            // [B][H/32][4 lanes-in-group][4 words] f16 fragments
  float* xscale;           // [B] power of 2 undoing the fragment pre-scale
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

// Upper bound on slots in one step: every pick its own slot, plus the shared expert's.
inline int max_slots(int B, int topk) {
  return B * topk + (B + DSMOE_SLOT_TOKENS - 1) / DSMOE_SLOT_TOKENS;
}

int launch_router(const RouterArgs& a, bool with_plan, cudaStream_t st);

}  // namespace dsmoe
