// Tensor-parallel group: device view of the symmetric NVLink buffers.
//
// Every rank owns one buffer with the same layout; peers write into it with
// plain P2P stores (CUDA IPC mappings).
//
// Row-parallel partials travel as 8-byte "LL" words, the fp32 value in the low
// half and the call's epoch in the high half, written with one 8-byte store:
// a reader that sees the epoch it waits for has the value too, so no fence or
// separate flag sits between a push and its use (the store's single-copy
// atomicity carries the ordering).  The LM-head key exchange (64-bit keys, no
// room for a tag) publishes with a release store of the epoch into a flag.
//
// Epochs come from a per-rank device counter (`state[kCalls]`) that the last
// CTA of every collective kernel advances, so the protocol needs no host
// argument per call and survives CUDA-graph replay.  Data slots alternate by
// epoch parity: a peer can be at most one call ahead (it cannot finish call
// e+1 before this rank has pushed call e+1, which happens after this rank
// finished reading call e), so parity e&1 is never overwritten while read.
// Flags compare with (int)(flag - epoch) >= 0 so a peer that already moved to
// the next epoch still satisfies the wait.
#pragma once

#include "common.cuh"

namespace jsx {

constexpr int kMaxRanks = 8;
constexpr int kMaxCtas = 1024;  // flag rows for per-CTA publication; row kMaxCtas is the LM-head row

enum { kCalls = 0, kDone = 1, kError = 2, kStateWords = 8 };

// Tile exchange of the wide row-parallel product (jsx_comm_create_tiles): an
// output tile of kXTileRows weight rows x kXTileTokens tokens is owned by rank
// (tile % world); the other ranks push their bf16 partial tiles into the
// owner's receive slots, the owner sums them in rank order, adds the residual
// and pushes the finished tile into every peer's result array.
constexpr int kXTileRows = 128;
constexpr int kXTileTokens = 256;
constexpr int kXQuarters = 4;  // flags per tile: one per epilogue warp (32 rows each)

struct CommDev {
  char* base[kMaxRanks];  // symmetric buffer of every rank, as mapped in this process
  uint32_t* state;        // local, not shared: calls, done, error
  int rank;
  int world;
  int max_tokens;
  int hidden;
  size_t off_data;        // u64 LL words [2][world][max_tokens][hidden]
  size_t off_keys;        // u64   [2][world][max_tokens]
  unsigned long long timeout_ns;
  // tile exchange (zero sizes unless created by jsx_comm_create_tiles)
  int max_tiles, max_owned;
  size_t off_pflags;      // u32 [max_owned][world][4]: partial (tile j, source, quarter) arrived
  size_t off_rflags;      // u32 [max_tiles][4]: finished tile quarter arrived
  size_t off_slots;       // bf16 [max_owned][world][4 quarters][256 tokens][32 rows]: partials
  size_t off_result;      // bf16 [max_tiles][4 quarters][256 tokens][32 rows]: finished tiles
};

__device__ __forceinline__ uint32_t* pflag_ptr(const CommDev& c, int r, int j, int src, int q) {
  return reinterpret_cast<uint32_t*>(c.base[r] + c.off_pflags) + ((size_t)j * c.world + src) * kXQuarters + q;
}
__device__ __forceinline__ uint32_t* rflag_ptr(const CommDev& c, int r, int tile, int q) {
  return reinterpret_cast<uint32_t*>(c.base[r] + c.off_rflags) + (size_t)tile * kXQuarters + q;
}
// [256 tokens][32 rows] block of quarter q (16 KB, contiguous)
__device__ __forceinline__ bf16* slot_ptr(const CommDev& c, int r, int j, int src, int q) {
  return reinterpret_cast<bf16*>(c.base[r] + c.off_slots) +
         (((size_t)j * c.world + src) * kXQuarters + q) * (kXTileTokens * kXTileRows / kXQuarters);
}
__device__ __forceinline__ bf16* result_ptr(const CommDev& c, int r, int tile, int q) {
  return reinterpret_cast<bf16*>(c.base[r] + c.off_result) +
         ((size_t)tile * kXQuarters + q) * (kXTileTokens * kXTileRows / kXQuarters);
}

// Bounded wait (every calling thread) until *f reaches `epoch`, with acquire
// at system scope; on timeout the comm's error word is set and false returned.
__device__ __forceinline__ bool wait_epoch_sys(const CommDev& c, const uint32_t* f, uint32_t epoch) {
  if ((int)(ld_acquire_sys(f) - epoch) >= 0) return true;
  if (*reinterpret_cast<volatile uint32_t*>(c.state + kError)) return false;
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    if ((int)(ld_acquire_sys(f) - epoch) >= 0) return true;
    if ((it & 63u) == 0) {
      if (globaltimer() - t0 > c.timeout_ns || it > (1u << 28)) {
        atomicOr(c.state + kError, 1u);
        return false;
      }
      __nanosleep(64);
    }
  }
}

__device__ __forceinline__ uint32_t* flag_ptr(const CommDev& c, int r, int row, int src) {
  return reinterpret_cast<uint32_t*>(c.base[r]) + (size_t)row * c.world + src;
}
__device__ __forceinline__ unsigned long long* data_ptr(const CommDev& c, int r, int par, int src, int m) {
  return reinterpret_cast<unsigned long long*>(c.base[r] + c.off_data) +
         ((size_t)(par * c.world + src) * c.max_tokens + m) * c.hidden;
}
__device__ __forceinline__ unsigned long long* key_ptr(const CommDev& c, int r, int par, int src) {
  return reinterpret_cast<unsigned long long*>(c.base[r] + c.off_keys) +
         (size_t)(par * c.world + src) * c.max_tokens;
}

__device__ __forceinline__ uint32_t read_epoch(const CommDev& c) {
  return *reinterpret_cast<volatile uint32_t*>(c.state + kCalls) + 1u;
}

// Bounded wait until this rank's flag (row, src) reaches `epoch`.  On timeout
// the error word is set and the caller proceeds (its output is then garbage
// and the host reports JSX_ETIMEDOUT through jsx_comm_check).
__device__ __forceinline__ void wait_flag(const CommDev& c, int row, int src, uint32_t epoch) {
  const uint32_t* f = flag_ptr(c, c.rank, row, src);
  const uint64_t t0 = globaltimer();
  uint32_t it = 0;
  while ((int)(ld_acquire_sys(f) - epoch) < 0) {
    ++it;
    if ((it & 63u) == 0) {
      if (globaltimer() - t0 > c.timeout_ns || it > (1u << 28)) {
        atomicOr(c.state + kError, 1u);
        return;
      }
    }
    __nanosleep(32);
  }
}

// Push one partial value to a peer's (or this rank's) slot.
__device__ __forceinline__ void ll_put(unsigned long long* slot, float v, uint32_t epoch) {
  const unsigned long long w = ((unsigned long long)epoch << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(slot), "l"(w) : "memory");
}

// The value of a slot once it carries `epoch`.  Bounded: after the comm
// timeout (or at once when an earlier wait of this rank gave up) the error
// word is set and 0 is returned; the host reports JSX_ETIMEDOUT.
__device__ __forceinline__ float ll_get(const CommDev& c, const unsigned long long* slot, uint32_t epoch) {
  unsigned long long w;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(slot) : "memory");
  if ((uint32_t)(w >> 32) == epoch) return __uint_as_float((uint32_t)w);
  if (*reinterpret_cast<volatile uint32_t*>(c.state + kError)) return 0.f;
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(slot) : "memory");
    if ((uint32_t)(w >> 32) == epoch) return __uint_as_float((uint32_t)w);
    if ((it & 15u) == 0) {
      if (globaltimer() - t0 > c.timeout_ns || it > (1u << 28)) {
        atomicOr(c.state + kError, 1u);
        return 0.f;
      }
      __nanosleep(20);
    }
  }
}

// Slow path of ll_sum_ranks (bounded by the comm timeout; on timeout the error
// word is set and a slot without the epoch counts as 0).
static __device__ __noinline__ float ll_sum_ranks_poll(const unsigned long long* p0, size_t sstride, int world,
                                                uint32_t* state, unsigned long long timeout_ns, uint32_t epoch) {
  // every slot still without the epoch is reloaded, all in flight together (one
  // round trip per pass), until all carry it; then the rank-ordered sum
  unsigned long long w[kMaxRanks];
#pragma unroll
  for (int src = 0; src < kMaxRanks; ++src) w[src] = 0ull;
  const uint64_t t0 = globaltimer();
  bool all = false;
#pragma unroll 1
  for (uint32_t it = 1; !all; ++it) {
#pragma unroll
    for (int src = 0; src < kMaxRanks; ++src)
      if (src < world && (uint32_t)(w[src] >> 32) != epoch)
        asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w[src]) : "l"(p0 + src * sstride) : "memory");
    all = true;
#pragma unroll
    for (int src = 0; src < kMaxRanks; ++src)
      if (src < world) all = all && (uint32_t)(w[src] >> 32) == epoch;
    if (!all && (it & 15u) == 0) {
      if (*reinterpret_cast<volatile uint32_t*>(state + kError)) break;
      if (globaltimer() - t0 > timeout_ns || it > (1u << 28)) {
        atomicOr(state + kError, 1u);
        break;
      }
      __nanosleep(20);
    }
  }
  float s = 0.f;
#pragma unroll
  for (int src = 0; src < kMaxRanks; ++src)
    if (src < world) s += (uint32_t)(w[src] >> 32) == epoch ? __uint_as_float((uint32_t)w[src]) : 0.f;
  return s;
}

// Sum in rank order of one value's LL slots (slot of rank src at p0 + src *
// sstride) once they carry `epoch`: every rank's slot is loaded before any is
// checked, so the sum costs one round trip when the pushes have landed.
__device__ __forceinline__ float ll_sum_ranks(const CommDev& c, const unsigned long long* p0, size_t sstride,
                                              uint32_t epoch) {
  unsigned long long w[kMaxRanks];
#pragma unroll
  for (int src = 0; src < kMaxRanks; ++src)
    if (src < c.world) asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w[src]) : "l"(p0 + src * sstride) : "memory");
  float s = 0.f;
  bool all = true;
#pragma unroll
  for (int src = 0; src < kMaxRanks; ++src) {
    if (src < c.world) {
      all = all && (uint32_t)(w[src] >> 32) == epoch;
      s += __uint_as_float((uint32_t)w[src]);
    }
  }
  return all ? s : ll_sum_ranks_poll(p0, sstride, c.world, c.state, c.timeout_ns, epoch);
}

}  // namespace jsx
