// Tensor-parallel group (utils/mesh_utils.py:8-45 "tensor" axis): one process
// per GPU, a symmetric buffer per rank shared through CUDA IPC, peer pointers
// used directly by the collective kernels (NVLink P2P stores).
#include <stdlib.h>
#include <string.h>

#include "comm.cuh"

struct jsx_comm {
  jsx::CommDev dev;
  char* local;
  size_t bytes;
  int device;
  bool opened;
};

namespace jsx {

CommDev comm_view(jsx_comm* comm) { return comm->dev; }

static size_t round256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace jsx

using namespace jsx;

namespace jsx {

// Allocates and zeroes the symmetric buffer (c->bytes, layout already set in
// c->dev) and the local state words.
static int comm_alloc(jsx_comm* c, jsx_comm** out) {
  JSX_CUDA(cudaGetDevice(&c->device));
  cudaError_t e = cudaMalloc((void**)&c->local, c->bytes);
  if (e != cudaSuccess) {
    free(c);
    return cuda_status(e, "cudaMalloc(symmetric buffer)");
  }
  e = cudaMalloc((void**)&c->dev.state, kStateWords * sizeof(uint32_t));
  if (e != cudaSuccess) {
    cudaFree(c->local);
    free(c);
    return cuda_status(e, "cudaMalloc(state)");
  }
  JSX_CUDA(cudaMemset(c->local, 0, c->bytes));
  JSX_CUDA(cudaMemset(c->dev.state, 0, kStateWords * sizeof(uint32_t)));
  JSX_CUDA(cudaDeviceSynchronize());
  c->dev.base[c->dev.rank] = c->local;
  c->opened = (c->dev.world == 1);
  *out = c;
  return JSX_OK;
}

static jsx_comm* comm_new(int rank, int world, int max_tokens, int hidden, uint64_t timeout_ns) {
  jsx_comm* c = (jsx_comm*)calloc(1, sizeof(jsx_comm));
  if (!c) return nullptr;
  c->dev.rank = rank;
  c->dev.world = world;
  c->dev.max_tokens = max_tokens;
  c->dev.hidden = hidden;
  c->dev.timeout_ns = timeout_ns ? timeout_ns : 5000000000ull;
  return c;
}

}  // namespace jsx

extern "C" int jsx_comm_create(int rank, int world, int max_tokens, int hidden, uint64_t timeout_ns,
                               jsx_comm** out) {
  JSX_REQUIRE(out != nullptr, "null out");
  JSX_REQUIRE(world >= 1 && world <= kMaxRanks, "world=%d outside 1..%d", world, kMaxRanks);
  JSX_REQUIRE(rank >= 0 && rank < world, "rank=%d outside [0, %d)", rank, world);
  JSX_REQUIRE(max_tokens >= 1 && max_tokens <= 4096, "max_tokens=%d", max_tokens);
  JSX_REQUIRE(hidden >= 1 && hidden <= (1 << 20), "hidden=%d", hidden);
  *out = nullptr;
  jsx_comm* c = comm_new(rank, world, max_tokens, hidden, timeout_ns);
  if (!c) {
    set_error("host allocation failed");
    return JSX_ENOMEM;
  }
  const size_t flags = round256((size_t)(kMaxCtas + 1) * world * sizeof(uint32_t));
  const size_t data = round256((size_t)2 * world * max_tokens * hidden * sizeof(unsigned long long));
  const size_t keys = round256((size_t)2 * world * max_tokens * sizeof(unsigned long long));
  c->bytes = flags + data + keys;
  c->dev.off_data = flags;
  c->dev.off_keys = flags + data;
  return comm_alloc(c, out);
}

extern "C" int jsx_comm_create_tiles(int rank, int world, int max_tokens, int hidden, uint64_t timeout_ns,
                                     jsx_comm** out) {
  JSX_REQUIRE(out != nullptr, "null out");
  JSX_REQUIRE(world >= 1 && world <= kMaxRanks, "world=%d outside 1..%d", world, kMaxRanks);
  JSX_REQUIRE(rank >= 0 && rank < world, "rank=%d outside [0, %d)", rank, world);
  JSX_REQUIRE(max_tokens >= 1 && max_tokens <= (1 << 20), "max_tokens=%d", max_tokens);
  JSX_REQUIRE(hidden >= 2 && hidden % 2 == 0 && hidden <= (1 << 20), "hidden=%d", hidden);
  *out = nullptr;
  jsx_comm* c = comm_new(rank, world, max_tokens, hidden, timeout_ns);
  if (!c) {
    set_error("host allocation failed");
    return JSX_ENOMEM;
  }
  const size_t tiles = (size_t)((max_tokens + kXTileTokens - 1) / kXTileTokens) *
                       ((hidden + kXTileRows - 1) / kXTileRows);
  const size_t owned = (tiles + world - 1) / world;
  const size_t pflags = round256(owned * world * kXQuarters * sizeof(uint32_t));
  const size_t rflags = round256(tiles * kXQuarters * sizeof(uint32_t));
  const size_t slots = round256(owned * world * kXTileTokens * kXTileRows * 2);
  const size_t result = round256(tiles * kXTileTokens * kXTileRows * 2);
  c->dev.max_tiles = (int)tiles;
  c->dev.max_owned = (int)owned;
  c->dev.off_pflags = 0;
  c->dev.off_rflags = pflags;
  c->dev.off_slots = pflags + rflags;
  c->dev.off_result = pflags + rflags + slots;
  c->bytes = pflags + rflags + slots + result;
  return comm_alloc(c, out);
}

extern "C" int jsx_comm_ipc_handle(jsx_comm* comm, void* out64) {
  JSX_REQUIRE(comm && out64, "null argument");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  cudaIpcMemHandle_t h;
  JSX_CUDA(cudaIpcGetMemHandle(&h, comm->local));
  memcpy(out64, &h, sizeof(h));
  return JSX_OK;
}

extern "C" int jsx_comm_open_peers(jsx_comm* comm, const void* handles) {
  JSX_REQUIRE(comm && handles, "null argument");
  JSX_REQUIRE(!comm->opened || comm->dev.world == 1, "peers already opened");
  for (int r = 0; r < comm->dev.world; ++r) {
    if (r == comm->dev.rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, (const char*)handles + 64 * (size_t)r, sizeof(h));
    void* p = nullptr;
    JSX_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    comm->dev.base[r] = (char*)p;
  }
  comm->opened = true;
  return JSX_OK;
}

extern "C" int jsx_comm_check(jsx_comm* comm, int* status) {
  JSX_REQUIRE(comm && status, "null argument");
  JSX_CUDA(cudaDeviceSynchronize());
  uint32_t err = 0;
  JSX_CUDA(cudaMemcpy(&err, comm->dev.state + kError, sizeof(err), cudaMemcpyDeviceToHost));
  if (err) {
    const uint32_t zero = 0;
    JSX_CUDA(cudaMemcpy(comm->dev.state + kError, &zero, sizeof(zero), cudaMemcpyHostToDevice));
  }
  *status = err ? JSX_ETIMEDOUT : JSX_OK;
  return JSX_OK;
}

extern "C" int jsx_comm_destroy(jsx_comm* comm) {
  if (!comm) return JSX_OK;
  cudaDeviceSynchronize();
  for (int r = 0; r < comm->dev.world; ++r)
    if (r != comm->dev.rank && comm->dev.base[r]) cudaIpcCloseMemHandle(comm->dev.base[r]);
  cudaFree(comm->local);
  cudaFree(comm->dev.state);
  free(comm);
  return JSX_OK;
}
