// Peer exchange for the all-reduce inside the persistent decode kernel: one device buffer per rank
// of the tensor-parallel group, mapped into every other rank's address space with CUDA IPC.
//
// It replaces the reference's per-layer `all_reduce_sum` (dsv41/tt/attn.py:19-21: all_gather of
// the 8 chips' partials over the ethernet mesh, then a sum), called after MoE.decode
// (dsv41/tt/moe.py:162, 180). Here the sum happens in the layer's own kernel: each rank stores its
// output-tile partials into its peers' buffers over NVLink and sums the tiles it receives (ar_tile
// in moe_fused.cu), so a layer is one launch on every rank with no collective library call.
//
// Set-up (host, once per group): every rank calls dsmoe_comm_create, the ranks exchange the
// 64-byte handles it returns (any host channel, e.g. an all-gather of the process group), then
// every rank calls dsmoe_comm_open with all handles in rank order.
#include <cstring>

#include "exchange.cuh"

struct dsmoe_comm {
  dsmoe::PeerExchange px;
  int device;
  size_t bytes;
  uint8_t* local;
  uint8_t* mapped[dsmoe::kMaxWorld];  // IPC mappings of the peers' buffers (nullptr for this rank)
  bool opened;
};

namespace dsmoe {
// Control region: word 0 = the epoch of the last call; word 1 = arrivals of the row all-reduce's
// CTAs; word 2 = status bits of the row all-reduce; words 4..7 = an identity {magic, world, hidden,
// bytes} that a peer checks before it maps the buffer; padded to keep the slots 256-byte aligned.
constexpr size_t kCtlBytes = 256;
constexpr unsigned kCommMagic = 0x64736D63u;  // "dsmc"
constexpr uint64_t kRowWaitNs = 5000000000ull;
constexpr unsigned CS_PEER = 1u;

// y[b][:] = sum over ranks of x[b][:] for b < B <= 8 tokens of `hidden` values (the reference's
// all_reduce_sum of the attention output projection, dsv41/tt/attn.py:19-21 at attn.py:229, 252).
// One warp per 16-row tile, the same lane layout and exchange as the decode kernel's output.
__global__ void allreduce_rows_kernel(PeerExchange px, const void* x, int x_f32, int B, void* y, int y_f32) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NT = px.hidden / 16, nt = blockIdx.x * (blockDim.x >> 5) + warp;
  __shared__ unsigned ep_s;
  if (threadIdx.x == 0) {
    ep_s = *(volatile unsigned*)px.ctl + 1u;
    __threadfence();  // the read of the old epoch precedes this CTA's arrival
    const unsigned old = atomicAdd(px.ctl + 1, 1u);
    if (old == gridDim.x - 1) {  // every CTA has read the old epoch: store the new one
      px.ctl[1] = 0u;
      __threadfence();
      *(volatile unsigned*)px.ctl = ep_s;
    }
  }
  __syncthreads();
  if (nt >= NT) return;
  const int g = lane >> 2, tq = lane & 3;
  float v[4];
#pragma unroll
  for (int q4 = 0; q4 < 4; ++q4) {
    const int row = nt * 16 + (q4 >= 2 ? g + 8 : g), tok = 2 * tq + (q4 & 1);
    const long long o = (long long)tok * px.hidden + row;
    v[q4] = tok >= B ? 0.f : x_f32 ? reinterpret_cast<const float*>(x)[o]
                                   : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[o]);
  }
  float4 s4 = make_float4(v[0], v[1], v[2], v[3]);
  if (!ll_allreduce_tile(px.slots, px.world, px.rank, NT, nt, B, ep_s, s4, lane, kRowWaitNs) && lane == 0)
    atomicOr(px.ctl + 2, CS_PEER);
  const float r[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
  for (int q4 = 0; q4 < 4; ++q4) {
    const int row = nt * 16 + (q4 >= 2 ? g + 8 : g), tok = 2 * tq + (q4 & 1);
    if (tok < B) {
      const long long o = (long long)tok * px.hidden + row;
      if (y_f32)
        reinterpret_cast<float*>(y)[o] = r[q4];
      else
        reinterpret_cast<__nv_bfloat16*>(y)[o] = __float2bfloat16_rn(r[q4]);
    }
  }
}
}

using namespace dsmoe;

extern "C" int dsmoe_comm_create(int rank, int world, int hidden, dsmoe_comm_t** out, void* handle_out) {
  DSMOE_REQUIRE(out && handle_out, DSMOE_ERR_ARG, "comm_create: out / handle_out null");
  *out = nullptr;
  DSMOE_REQUIRE(world >= 2 && world <= kMaxWorld, DSMOE_ERR_ARG, "comm_create: world %d outside 2..%d", world,
                kMaxWorld);
  DSMOE_REQUIRE(rank >= 0 && rank < world, DSMOE_ERR_ARG, "comm_create: rank %d outside 0..%d", rank, world - 1);
  DSMOE_REQUIRE(hidden > 0 && hidden % 16 == 0, DSMOE_ERR_ARG, "comm_create: hidden %d must be a multiple of 16",
                hidden);
  dsmoe_comm* c = new dsmoe_comm();
  std::memset(c, 0, sizeof(*c));
  if (cudaGetDevice(&c->device) != cudaSuccess) {
    delete c;
    return cuda_status("comm_create: cudaGetDevice");
  }
  c->bytes = kCtlBytes + exchange_slot_words(world, hidden) * 8;
  void* p = nullptr;
  if (cudaMalloc(&p, c->bytes) != cudaSuccess) {
    delete c;
    return cuda_status("comm_create: cudaMalloc");
  }
  c->local = (uint8_t*)p;
  // epoch 0 and all-zero slots: no word carries an epoch of a call yet (epochs start at 1)
  if (cudaMemset(p, 0, c->bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(p);
    delete c;
    return cuda_status("comm_create: clear");
  }
  const unsigned ident[4] = {kCommMagic, (unsigned)world, (unsigned)hidden, (unsigned)c->bytes};
  if (cudaMemcpy((uint8_t*)p + 16, ident, sizeof(ident), cudaMemcpyHostToDevice) != cudaSuccess) {
    cudaFree(p);
    delete c;
    return cuda_status("comm_create: identity");
  }
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    delete c;
    return cuda_status("comm_create: cudaIpcGetMemHandle");
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == DSMOE_COMM_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle_out, &h, sizeof(h));
  c->px.rank = rank;
  c->px.world = world;
  c->px.hidden = hidden;
  c->px.ctl = (unsigned*)c->local;
  c->px.slots[rank] = (unsigned long long*)(c->local + kCtlBytes);
  *out = c;
  return DSMOE_OK;
}

extern "C" int dsmoe_comm_open(dsmoe_comm_t* c, const void* handles) {
  DSMOE_REQUIRE(c && handles, DSMOE_ERR_ARG, "comm_open: comm / handles null");
  DSMOE_REQUIRE(!c->opened, DSMOE_ERR_ARG, "comm_open: already open");
  int dev = -1;
  cudaGetDevice(&dev);
  DSMOE_REQUIRE(dev == c->device, DSMOE_ERR_ARG, "comm_open: device %d current, comm created on %d", dev, c->device);
  const uint8_t* hs = (const uint8_t*)handles;
  for (int q = 0; q < c->px.world; ++q) {
    if (q == c->px.rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, hs + (size_t)q * DSMOE_COMM_HANDLE_BYTES, sizeof(h));
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      const int rc = cuda_status("comm_open: cudaIpcOpenMemHandle");
      for (int j = 0; j < q; ++j)
        if (c->mapped[j]) {
          cudaIpcCloseMemHandle(c->mapped[j]);
          c->mapped[j] = nullptr;
          c->px.slots[j] = nullptr;
        }
      return rc;
    }
    c->mapped[q] = (uint8_t*)p;
    // the peer's buffer must have this rank's geometry: every store into it stays inside
    unsigned ident[4] = {0, 0, 0, 0};
    const bool read = cudaMemcpy(ident, (uint8_t*)p + 16, sizeof(ident), cudaMemcpyDeviceToHost) == cudaSuccess;
    if (!read || ident[0] != kCommMagic || ident[1] != (unsigned)c->px.world || ident[2] != (unsigned)c->px.hidden ||
        ident[3] != (unsigned)c->bytes) {
      if (!read) cudaGetLastError();
      for (int j = 0; j <= q; ++j)
        if (c->mapped[j]) {
          cudaIpcCloseMemHandle(c->mapped[j]);
          c->mapped[j] = nullptr;
          c->px.slots[j] = nullptr;
        }
      set_error("comm_open: rank %d's exchange buffer is not a comm of world %d, hidden %d (read %s)", q,
                c->px.world, c->px.hidden, read ? "ok" : "failed");
      return DSMOE_ERR_ARG;
    }
    c->px.slots[q] = (unsigned long long*)((uint8_t*)p + kCtlBytes);
  }
  c->opened = true;
  return DSMOE_OK;
}

extern "C" int dsmoe_comm_destroy(dsmoe_comm_t* c) {
  if (!c) return DSMOE_OK;
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != c->device) cudaSetDevice(c->device);
  cudaDeviceSynchronize();
  for (int q = 0; q < kMaxWorld; ++q)
    if (c->mapped[q]) cudaIpcCloseMemHandle(c->mapped[q]);
  if (c->local) cudaFree(c->local);
  if (prev >= 0 && prev != c->device) cudaSetDevice(prev);
  delete c;
  return cuda_status("comm_destroy");
}

namespace dsmoe {
const PeerExchange* comm_exchange(const dsmoe_comm_t* c) { return c && c->opened ? &c->px : nullptr; }
}  // namespace dsmoe

extern "C" int dsmoe_allreduce_rows(const dsmoe_comm_t* c, const void* x, int x_dtype, int B, void* y, int y_dtype,
                                    void* stream) {
  DSMOE_REQUIRE(c && c->opened, DSMOE_ERR_ARG, "allreduce_rows: comm is null or not opened");
  DSMOE_REQUIRE(x && y, DSMOE_ERR_ARG, "allreduce_rows: x / y null");
  DSMOE_REQUIRE(B >= 1 && B <= 8, DSMOE_ERR_ARG, "allreduce_rows: rows %d outside 1..8", B);
  DSMOE_REQUIRE((x_dtype == DSMOE_DTYPE_BF16 || x_dtype == DSMOE_DTYPE_F32) &&
                    (y_dtype == DSMOE_DTYPE_BF16 || y_dtype == DSMOE_DTYPE_F32),
                DSMOE_ERR_ARG, "allreduce_rows: dtypes %d -> %d", x_dtype, y_dtype);
  int dev = -1;
  cudaGetDevice(&dev);
  DSMOE_REQUIRE(dev == c->device, DSMOE_ERR_ARG, "allreduce_rows: device %d current, comm on %d", dev, c->device);
  const int NT = c->px.hidden / 16, wpb = 8;
  allreduce_rows_kernel<<<(NT + wpb - 1) / wpb, wpb * 32, 0, (cudaStream_t)stream>>>(
      c->px, x, x_dtype == DSMOE_DTYPE_F32, B, y, y_dtype == DSMOE_DTYPE_F32);
  return cuda_status("allreduce_rows");
}

extern "C" int dsmoe_comm_check(const dsmoe_comm_t* c, void* stream) {
  DSMOE_REQUIRE(c, DSMOE_ERR_ARG, "comm_check: comm is null");
  if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) return cuda_status("comm_check: synchronize");
  unsigned st = 0;
  if (cudaMemcpy(&st, c->local + 8, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return cuda_status("comm_check: read");
  if (st == 0) return DSMOE_OK;
  cudaMemset(c->local + 8, 0, 4);
  set_error("allreduce_rows: a peer's tile did not arrive within the bound (status 0x%x); re-create the comm", st);
  return DSMOE_ERR_TIMEOUT;
}
