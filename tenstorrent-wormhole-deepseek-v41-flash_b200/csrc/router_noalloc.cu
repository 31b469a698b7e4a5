// dsmoe_router without a caller workspace: the same router kernels (router.cu), with their scratch
// in one file-scope device array instead of caller-provided memory.
//
// Who needs it: callers that cannot hand the library device memory for scratch. Examples are a
// language binding with no device allocator of its own (a C or Go host that only owns the input
// and output buffers), and a serving loop that must not allocate after start-up, where a
// cudaMalloc would synchronise the device and torch's caching allocator is not available. For them
// the scratch lives in this library's image; nothing is allocated at any call.
//
// Limits: B <= 64 tokens, E <= 1024 experts, hidden <= 8192, top-k <= 8. The array holds
// logits [B][E] fp32, the top-k [B][k] as int32 and fp32, the token rows in e4m3 hi / lo form
// [B][2][hidden] and one fp32 pre-scale per token, each region 256-byte aligned, sized for those
// maxima (1,315,072 bytes). Larger calls are rejected with DSMOE_ERR_ARG.
// Nothing in the array needs to start at zero: every word a call reads was written earlier in the
// same call.
// One array per device (one module instance per device context) serves every call on that device,
// so calls on one device must not overlap: overlapping calls (two streams, or two host threads)
// race on the scratch. Serialise them on one stream.
// Set-up: the first call on a device, with that device current, looks up the array's address with
// cudaGetSymbolAddress and keeps it; that first call must come before any stream capture.
#include <mutex>

#include "router.cuh"

namespace dsmoe {

constexpr int kNaMaxB = 64, kNaMaxE = 1024, kNaMaxH = 8192, kNaMaxK = DSMOE_MAX_TOPK;
constexpr size_t na_al(size_t v) { return (v + 255) & ~size_t(255); }
constexpr size_t kNaLogits = 0;
constexpr size_t kNaIdx = kNaLogits + na_al((size_t)kNaMaxB * kNaMaxE * 4);
constexpr size_t kNaWt = kNaIdx + na_al((size_t)kNaMaxB * kNaMaxK * 4);
constexpr size_t kNaXq = kNaWt + na_al((size_t)kNaMaxB * kNaMaxK * 4);
constexpr size_t kNaXscale = kNaXq + na_al((size_t)kNaMaxB * 2 * kNaMaxH);
constexpr size_t kNaScratchBytes = kNaXscale + na_al((size_t)kNaMaxB * 4);
static_assert(kNaScratchBytes == 1315072, "stated scratch size");

static __device__ __align__(256) uint8_t g_router_scratch[kNaScratchBytes];

static void* g_scratch_ptr[64];
static std::mutex g_scratch_mu;

// The array's device address on the current device, looked up once per device.
static int router_scratch(uint8_t** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cuda_status("router_noalloc: cudaGetDevice");
  DSMOE_REQUIRE(dev >= 0 && dev < 64, DSMOE_ERR_UNSUPPORTED, "router_noalloc: device %d beyond 64", dev);
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_router_scratch);
    if (e != cudaSuccess || !p) {
      cudaGetLastError();
      set_error("router_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return DSMOE_ERR_CUDA;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = static_cast<uint8_t*>(g_scratch_ptr[dev]);
  return DSMOE_OK;
}

}  // namespace dsmoe

using namespace dsmoe;

extern "C" int dsmoe_router_noalloc(const dsmoe_layer_t* L, const void* x, int B, const uint8_t* image_mask,
                                    int64_t* idx, float* wt, float* scores, void* stream) {
  DSMOE_REQUIRE(L, DSMOE_ERR_ARG, "router_noalloc: layer is null");
  DSMOE_REQUIRE(B >= 1 && B <= kNaMaxB, DSMOE_ERR_ARG, "router_noalloc: batch %d outside 1..%d (scratch limit)", B,
                kNaMaxB);
  DSMOE_REQUIRE(L->hidden > 0 && L->hidden % 128 == 0 && L->hidden <= kNaMaxH, DSMOE_ERR_ARG,
                "router_noalloc: hidden %d must be a multiple of 128 and <= %d (scratch limit)", L->hidden, kNaMaxH);
  DSMOE_REQUIRE(L->n_experts >= 1 && L->n_experts <= kNaMaxE, DSMOE_ERR_ARG,
                "router_noalloc: n_experts %d outside 1..%d (scratch limit)", L->n_experts, kNaMaxE);
  DSMOE_REQUIRE(L->topk >= 1 && L->topk <= kNaMaxK && L->topk <= L->n_experts, DSMOE_ERR_ARG,
                "router_noalloc: topk %d outside 1..min(%d, n_experts)", L->topk, kNaMaxK);
  DSMOE_REQUIRE(L->score_func == DSMOE_SCORE_SIGMOID || L->score_func == DSMOE_SCORE_SQRTSOFTPLUS, DSMOE_ERR_ARG,
                "router_noalloc: score_func %d", L->score_func);
  DSMOE_REQUIRE(L->gate_w && L->gate_bias && x && idx && wt, DSMOE_ERR_ARG,
                "router_noalloc: gate_w / gate_bias / x / idx / wt must not be null");
  DSMOE_REQUIRE(((uintptr_t)L->gate_w & 15) == 0 && ((uintptr_t)x & 7) == 0, DSMOE_ERR_ALIGN,
                "router_noalloc: gate_w must be 16-byte and x 8-byte aligned");
  uint8_t* s = nullptr;
  const int rc = router_scratch(&s);
  if (rc) return rc;

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
  a.logits = reinterpret_cast<float*>(s + kNaLogits);
  a.idx32 = reinterpret_cast<int*>(s + kNaIdx);
  a.wt32 = reinterpret_cast<float*>(s + kNaWt);
  a.xq = s + kNaXq;
  a.xscale = reinterpret_cast<float*>(s + kNaXscale);
  a.idx = idx;
  a.wt = wt;
  a.scores = scores;
  return launch_router(a, false, (cudaStream_t)stream);
}
