// Decode GEMV family (M <= 8 tokens): the weight-streaming kernels of one
// GLM-4 decoder step, each with its prologue/epilogue fused.
//
//   jsx_linear                 LinearBase (layers/linear.py:57-82), optional RMSNorm prologue
//   jsx_qkv_rope_cache         input_layernorm + q/k/v + bias + RoPE + KV-cache write
//   jsx_gate_up_swiglu         post_attention_layernorm + gate/up + SwiGLU
//   jsx_row_linear_allreduce   o_proj/down_proj + TP all-reduce (NVLink P2P) + residual
//   jsx_lmhead_argmax          final norm + LM head + greedy argmax (+ cross-rank argmax)
//
// Layout: weights are packed row-major [N_rows][K] (each output row's K inputs
// contiguous), so a warp streams whole 512-byte lines with 16-byte
// non-allocating loads.  The activations (M x K bf16, optionally RMS-
// normalised) are staged once per CTA in shared memory.
//
// Work split: rows are processed in groups of kRows by one warp; group g goes
// to CTA g % grid so that every SM gets work even when the row count is small
// (o_proj/down at N = 4096).  The grid is persistent (<= resident CTAs), which
// the peer protocol of the row-parallel kernel relies on: every CTA of every
// rank is resident, so a CTA that waits for its peers never blocks a CTA they
// wait for.
//
// Programmatic dependent launch: each kernel issues its first weight loads
// BEFORE griddepcontrol.wait (weights never depend on the previous kernel) and
// performs every activation read and every global write after it.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "comm.cuh"
#include "common.cuh"
#include "gemv_core.cuh"
#include "launch.cuh"

namespace jsx {

// ---- the kernel ------------------------------------------------------------------
template <int M, int EPI>
__global__ void __launch_bounds__(kThreads) k_gemv(GemvArgs a, CommDev c) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  bf16* xs = reinterpret_cast<bf16*>(smem_raw);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nvec = a.K >> 3;
  const int ngroups = a.N / kRows;
  const int grid = gridDim.x;
  const uint4* wbase = reinterpret_cast<const uint4*>(a.w);
  const size_t group_vecs = (size_t)kRows * nvec;

  int g = blockIdx.x + grid * warp;
  Batch bt;
  if (g < ngroups) load_batch(bt, wbase + (size_t)g * group_vecs, nvec, 0, lane);

  pdl_wait();
  pdl_launch_dependents();

  const bool multi = (EPI == EPI_ROWAR || EPI == EPI_LMHEAD) && c.world > 1;
  uint32_t epoch = 0;
  if (EPI == EPI_ROWAR && multi) epoch = read_epoch(c);

  stage_x<M>(a, xs);
  const uint4* xv = reinterpret_cast<const uint4*>(xs);

  unsigned long long best[M];
#pragma unroll
  for (int m = 0; m < M; ++m) best[m] = 0ull;

  for (; g < ngroups; g += grid * kWarps) {
    const uint4* wv = wbase + (size_t)g * group_vecs;
    float acc[kRows][M];
#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
      for (int m = 0; m < M; ++m) acc[r][m] = 0.f;

    for (int base = 0; base < nvec; base += 32 * kUnroll) {
      if (base > 0) load_batch(bt, wv, nvec, base, lane);
      fma_batch<M>(bt, xv, nvec, base, lane, acc);
    }
    // Prefetch the next group's first batch before the reductions/epilogue.
    const int gn = g + grid * kWarps;
    if (gn < ngroups) load_batch(bt, wbase + (size_t)gn * group_vecs, nvec, 0, lane);

#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
      for (int m = 0; m < M; ++m) acc[r][m] = warp_sum(acc[r][m]);

    if constexpr (EPI == EPI_LINEAR) {
      if (lane < kRows * M) {
        const int r = lane / M, m = lane - (lane / M) * M;
        const int row = g * kRows + r;
        float v = rbf(pick<M>(acc, r, m));
        if (a.bias) v = rbf(v + ldbf(a.bias + row));
        a.y[(size_t)m * a.N + row] = __float2bfloat16_rn(v);
      }
    } else if constexpr (EPI == EPI_QKV) {
      epi_qkv<M>(a, g, acc, lane);
    } else if constexpr (EPI == EPI_SWIGLU) {
      epi_swiglu<M>(a, g, acc, lane);
    } else if constexpr (EPI == EPI_ROWAR) {
      if (lane < kRows * M) {
        const int r = lane / M, m = lane - (lane / M) * M;
        const int row = g * kRows + r;
        float v = pick<M>(acc, r, m);
        if (a.addend) v += ldbf(a.addend + (size_t)m * a.N + row);
        if (!multi) {
          bf16* hp = a.h + (size_t)m * a.N + row;
          *hp = __float2bfloat16_rn(__bfloat162float(*hp) + rbf(v));
        } else {
          for (int d = 0; d < c.world; ++d) ll_put(data_ptr(c, d, epoch & 1, c.rank, m) + row, v, epoch);
        }
      }
    } else if constexpr (EPI == EPI_LMHEAD) {
      // logits are bf16 in the reference (layers/embedding.py:88-92)
      unsigned long long key = 0ull;
      int mine = -1;
      if (lane < kRows * M) {
        const int r = lane / M, m = lane - (lane / M) * M;
        const int row = g * kRows + r;
        const float v = rbf(pick<M>(acc, r, m));
        if (a.y) a.y[(size_t)m * a.N + row] = __float2bfloat16_rn(v);
        key = argmax_key(v, (uint32_t)(a.vocab_offset + row));
        mine = m;
      }
#pragma unroll
      for (int m = 0; m < M; ++m) {
        unsigned long long k = warp_max_u64(mine == m ? key : 0ull);
        best[m] = k > best[m] ? k : best[m];
      }
    }
  }

  if constexpr (EPI == EPI_ROWAR) {
    if (multi) {
      // gather this CTA's rows from every rank's LL slots (rank order)
      const int my_groups = (ngroups - (int)blockIdx.x + grid - 1) / grid;
      const int entries = my_groups * kRows * M;
      for (int e = threadIdx.x; e < entries; e += blockDim.x) {
        const int gl = e / (kRows * M);
        const int rem = e - gl * kRows * M;
        const int r = rem / M, m = rem - (rem / M) * M;
        const int row = (blockIdx.x + grid * gl) * kRows + r;
        const float s = ll_sum_ranks(c, data_ptr(c, c.rank, epoch & 1, 0, m) + row, (size_t)c.max_tokens * c.hidden,
                                     epoch);
        bf16* hp = a.h + (size_t)m * a.N + row;
        *hp = __float2bfloat16_rn(__bfloat162float(*hp) + rbf(s));
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        if (atomicAdd(c.state + kDone, 1u) == gridDim.x - 1) {
          c.state[kDone] = 0u;
          __threadfence();
          c.state[kCalls] = epoch;
        }
      }
    }
  }

  if constexpr (EPI == EPI_LMHEAD) {
    __shared__ unsigned long long cta_best[kWarps][M];
    __shared__ bool is_last;
    if (lane == 0) {
#pragma unroll
      for (int m = 0; m < M; ++m) cta_best[warp][m] = best[m];
    }
    __syncthreads();
    if (threadIdx.x < M) {
      unsigned long long b = 0ull;
      for (int w = 0; w < kWarps; ++w) b = cta_best[w][threadIdx.x] > b ? cta_best[w][threadIdx.x] : b;
      atomicMax(a.keys + threadIdx.x, b);
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) is_last = atomicAdd(a.done, 1u) == gridDim.x - 1;
    __syncthreads();
    if (is_last) {
      __threadfence();
      __shared__ unsigned long long fin[M];
      if (threadIdx.x < M) fin[threadIdx.x] = atomicAdd(a.keys + threadIdx.x, 0ull);
      __syncthreads();
      if (multi) {
        const uint32_t ep = read_epoch(c);
        const int pr = ep & 1;
        if (threadIdx.x < M)
          for (int d = 0; d < c.world; ++d) key_ptr(c, d, pr, c.rank)[threadIdx.x] = fin[threadIdx.x];
        __threadfence_system();
        __syncthreads();
        if (threadIdx.x < c.world) st_release_sys(flag_ptr(c, threadIdx.x, kMaxCtas, c.rank), ep);
        if (threadIdx.x < c.world) wait_flag(c, kMaxCtas, threadIdx.x, ep);
        __syncthreads();
        if (threadIdx.x < M) {
          unsigned long long b = 0ull;
          for (int s = 0; s < c.world; ++s) {
            const unsigned long long k = __ldcg(key_ptr(c, c.rank, pr, s) + threadIdx.x);
            b = k > b ? k : b;
          }
          fin[threadIdx.x] = b;
        }
        __syncthreads();
        if (threadIdx.x == 0) c.state[kCalls] = ep;
      }
      if (threadIdx.x < M) {
        a.ids[threadIdx.x] = (int32_t)argmax_key_index(fin[threadIdx.x]);
        a.keys[threadIdx.x] = 0ull;
      }
      if (threadIdx.x == 0) *a.done = 0u;
    }
  }
}

// ---- streaming kernel: weights through shared memory (cp.async.bulk) --------------
// One CTA per SM: 8 consumer warps + 1 producer warp.  The CTA owns a
// contiguous range of row pairs (packed rows 2b, 2b+1), split evenly to within
// one pair.  An "item" is nb consecutive pairs (nb > 1 only for K <= 2048, so
// that a stage carries >= 8 KB); items are dealt round-robin to the consumer
// warps and every warp owns its items end to end: it accumulates both rows of
// a pair over the K chunks, reduces inside the warp and runs the pair's
// epilogue itself, so the main loop has no CTA-wide barrier.
//
// The producer warp's elected lane streams the units (one K chunk of one item,
// <= 16 KB) into a ring of shared-memory stages with cp.async.bulk (L2
// evict-first), in the order (group of 8 items, chunk, item) so the eight warps
// are fed in turn; each stage completes on a full mbarrier (expect_tx) and is
// handed back by its warp on an empty mbarrier.  The producer never reads
// activations, so it skips griddepcontrol.wait and keeps loading weights while
// the previous kernel drains.  Bytes in flight per SM = stages x 16 KB.
//
// Every wait is time-bounded; on a timeout the CTA raises an abort flag and the
// device error word, warps stop waiting (they still hand back their stages),
// and the producer drains the copies it issued before it exits.
constexpr int kMaxStages = 48;
constexpr int kMinStages = 12;
constexpr int kConsumers = 8;
constexpr int kStreamThreads = (kConsumers + 1) * 32;
constexpr long long kWaitLimitCycles = 4000000000ll;

static __device__ uint32_t g_gemv_error;  // read and cleared by jsx_device_error

struct StreamPlan {
  int stage_bytes;  // bytes per stage (4, 8 or 16 KB)
  int nb;      // row pairs per item (1, 2 or 4)
  int Kc;      // chunk length in elements (K when nchunk == 1)
  int nchunk;  // chunks per item
  int stages;
  int x_bytes; // shared bytes of the staged activations (16-byte multiple)
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase of parity `parity` to complete.  Returns false
// (without waiting) once the CTA has aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, volatile int* abort) {
  if (*abort) return false;
  if (mbar_try_wait(b, parity)) return true;
  // bound on the SM cycle counter (cheap to read): kWaitLimitCycles ~ 2 s at the 1965 MHz max clock
  const long long t0 = clock64();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(b, parity)) return true;
    if ((it & 63u) == 0) {
      if (*abort) return false;
      if (clock64() - t0 > kWaitLimitCycles) {
        *abort = 1;
        atomicOr(&g_gemv_error, 1u);
        return false;
      }
    }
  }
}
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                          uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

template <int M, int EPI>
__global__ void __launch_bounds__(kStreamThreads, 1) k_gemv_stream(GemvArgs a, CommDev c, StreamPlan pl) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char* stages = smem_raw;
  bf16* xs = reinterpret_cast<bf16*>(smem_raw + (size_t)pl.stages * pl.stage_bytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw + (size_t)pl.stages * pl.stage_bytes + pl.x_bytes);
  uint64_t* empty = full + pl.stages;
  __shared__ int abort_flag;
  __shared__ bool is_last;
  __shared__ unsigned long long cta_best[kConsumers][M];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = a.K;
  const int NB = a.N >> 1;  // row pairs
  const int b0 = (int)((long long)blockIdx.x * NB / gridDim.x);
  const int b1 = (int)((long long)(blockIdx.x + 1) * NB / gridDim.x);
  const int nitems = (b1 - b0 + pl.nb - 1) / pl.nb;
  const int units = nitems * pl.nchunk;
  const int group_units = kConsumers * pl.nchunk;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < pl.stages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    mbar_fence_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kConsumers) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint64_t policy = l2_evict_first();
      int u = 0;
      for (; u < units; ++u) {
        const int s = u % pl.stages, i = u / pl.stages;
        if (i > 0 && !mbar_wait(empty + s, (i - 1) & 1, &abort_flag)) break;
        const int gi = u / group_units, o = u - gi * group_units;
        const int gsz = min(kConsumers, nitems - gi * kConsumers);
        const int ch = o / gsz, item = gi * kConsumers + (o - ch * gsz);
        const int p0 = b0 + item * pl.nb, np = min(pl.nb, b1 - p0);
        const int k0 = ch * pl.Kc, kl = min(pl.Kc, K - k0);
        unsigned char* dst = stages + (size_t)s * pl.stage_bytes;
        if (pl.nchunk == 1) {
          const uint32_t bytes = (uint32_t)np * 4u * (uint32_t)K;  // 2 np rows, contiguous
          mbar_expect_tx(full + s, bytes);
          bulk_load(dst, a.w + (size_t)p0 * 2 * K, bytes, full + s, policy);
        } else {
          const uint32_t bytes = (uint32_t)kl * 2u;
          mbar_expect_tx(full + s, 2u * bytes);
          bulk_load(dst, a.w + (size_t)(2 * p0) * K + k0, bytes, full + s, policy);
          bulk_load(dst + bytes, a.w + (size_t)(2 * p0 + 1) * K + k0, bytes, full + s, policy);
        }
      }
      // Drain: every copy issued must land before this CTA can exit.
      volatile int no_abort = 0;
      const int first = u > pl.stages ? u - pl.stages : 0;
      for (int v = first; v < u; ++v) mbar_wait(full + v % pl.stages, (v / pl.stages) & 1, &no_abort);
    }
    return;
  }

  // ---------------- consumers ----------------
  pdl_wait();
  const bool multi = (EPI == EPI_ROWAR || EPI == EPI_LMHEAD) && c.world > 1;
  uint32_t epoch = 0;
  if (EPI == EPI_ROWAR && multi) epoch = read_epoch(c);
  stage_x<M, true>(a, xs);

  const uint4* xv = reinterpret_cast<const uint4*>(xs);
  const int xstride = K >> 3;
  unsigned long long best = 0ull;
  float acc[kRows][M];
  // acc += both rows of one pair over kl columns starting at k0 (stage rows w0, w1)
  auto accumulate = [&](const unsigned char* pair_base, int kl, int k0) {
    const uint4* w0 = reinterpret_cast<const uint4*>(pair_base);
    const uint4* w1 = reinterpret_cast<const uint4*>(pair_base + (size_t)kl * 2);
    const int kv = kl >> 3, xo = k0 >> 3;
    for (int v = lane; v < kv; v += 32) {
      float f0[8], f1[8];
      unpack8(w0[v], f0);
      unpack8(w1[v], f1);
#pragma unroll
      for (int m = 0; m < M; ++m) {
        float xf[8];
        unpack8(xv[m * xstride + xo + v], xf);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          acc[0][m] = fmaf(f0[j], xf[j], acc[0][m]);
          acc[1][m] = fmaf(f1[j], xf[j], acc[1][m]);
        }
      }
    }
  };
  auto zero = [&]() {
#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
      for (int m = 0; m < M; ++m) acc[r][m] = 0.f;
  };
  auto finish_pair = [&](int pair, bool ok) {
#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
      for (int m = 0; m < M; ++m) acc[r][m] = warp_sum(acc[r][m]);
    if (ok && lane < M && !abort_flag) {
      const unsigned long long k =
          epi_pair<EPI>(a, c, multi, epoch, pair, lane, pick<M>(acc, 0, lane), pick<M>(acc, 1, lane));
      best = k > best ? k : best;
    }
  };

  for (int gi = 0; gi * kConsumers < nitems; ++gi) {
    const int gsz = min(kConsumers, nitems - gi * kConsumers);
    if (warp >= gsz) break;
    const int item = gi * kConsumers + warp;
    const int p0 = b0 + item * pl.nb, np = min(pl.nb, b1 - p0);
    if (pl.nchunk == 1) {
      // one stage holds the item's np whole pairs
      const int u = gi * group_units + warp, s = u % pl.stages;
      const bool ok = mbar_wait(full + s, (u / pl.stages) & 1, &abort_flag);
      const unsigned char* st = stages + (size_t)s * pl.stage_bytes;
      for (int pp = 0; pp < np; ++pp) {
        zero();
        if (ok) accumulate(st + (size_t)pp * 4 * K, K, 0);
        if (pp == np - 1) {
          __syncwarp();
          if (lane == 0) mbar_arrive(empty + s);
        }
        finish_pair(p0 + pp, ok);
      }
    } else {
      // one pair, one K chunk per stage
      zero();
      bool ok_all = true;
      for (int ch = 0; ch < pl.nchunk; ++ch) {
        const int u = gi * group_units + ch * gsz + warp, s = u % pl.stages;
        const bool ok = mbar_wait(full + s, (u / pl.stages) & 1, &abort_flag);
        const int k0 = ch * pl.Kc, kl = min(pl.Kc, K - k0);
        if (ok) accumulate(stages + (size_t)s * pl.stage_bytes, kl, k0);
        ok_all = ok_all && ok;
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + s);
      }
      finish_pair(p0, ok_all);
    }
  }

  if constexpr (EPI == EPI_ROWAR) {
    if (multi) {
      const int rows = 2 * (b1 - b0);
      for (int e = threadIdx.x; e < rows * M; e += kThreads) {
        const int m = e / rows, row = 2 * b0 + (e - (e / rows) * rows);
        const float sum = ll_sum_ranks(c, data_ptr(c, c.rank, epoch & 1, 0, m) + row,
                                       (size_t)c.max_tokens * c.hidden, epoch);
        bf16* hp = a.h + (size_t)m * a.N + row;
        *hp = __float2bfloat16_rn(__bfloat162float(*hp) + rbf(sum));
      }
      consumer_sync();
      if (threadIdx.x == 0) {
        if (atomicAdd(c.state + kDone, 1u) == gridDim.x - 1) {
          c.state[kDone] = 0u;
          __threadfence();
          c.state[kCalls] = epoch;
        }
      }
    }
  }

  if constexpr (EPI == EPI_LMHEAD) {
    // lane m < M of every warp holds that warp's best key for token m
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const unsigned long long k = __shfl_sync(0xffffffffu, best, m);
      if (lane == 0) cta_best[warp][m] = k;
    }
    consumer_sync();
    if (threadIdx.x < M) {
      unsigned long long b = 0ull;
      for (int w = 0; w < kConsumers; ++w) b = cta_best[w][threadIdx.x] > b ? cta_best[w][threadIdx.x] : b;
      if (b) atomicMax(a.keys + threadIdx.x, b);
    }
    __threadfence();
    consumer_sync();
    if (threadIdx.x == 0) is_last = atomicAdd(a.done, 1u) == gridDim.x - 1;
    consumer_sync();
    if (is_last) {
      __threadfence();
      __shared__ unsigned long long fin[M];
      if (threadIdx.x < M) fin[threadIdx.x] = atomicAdd(a.keys + threadIdx.x, 0ull);
      consumer_sync();
      if (multi) {
        const uint32_t ep = read_epoch(c);
        const int pr = ep & 1;
        if (threadIdx.x < M)
          for (int d = 0; d < c.world; ++d) key_ptr(c, d, pr, c.rank)[threadIdx.x] = fin[threadIdx.x];
        __threadfence_system();
        consumer_sync();
        if (threadIdx.x < c.world) st_release_sys(flag_ptr(c, threadIdx.x, kMaxCtas, c.rank), ep);
        if (threadIdx.x < c.world) wait_flag(c, kMaxCtas, threadIdx.x, ep);
        consumer_sync();
        if (threadIdx.x < M) {
          unsigned long long b = 0ull;
          for (int sx = 0; sx < c.world; ++sx) {
            const unsigned long long k = __ldcg(key_ptr(c, c.rank, pr, sx) + threadIdx.x);
            b = k > b ? k : b;
          }
          fin[threadIdx.x] = b;
        }
        consumer_sync();
        if (threadIdx.x == 0) c.state[kCalls] = ep;
      }
      if (threadIdx.x < M) {
        a.ids[threadIdx.x] = (int32_t)argmax_key_index(fin[threadIdx.x]);
        a.keys[threadIdx.x] = 0ull;
      }
      if (threadIdx.x == 0) *a.done = 0u;
    }
  }
}

// ---- host side ---------------------------------------------------------------------
// JSX_GEMV=stream selects the shared-memory streaming kernel wherever its
// stages fit.  Default: the register-streaming kernel, which measured faster on
// B200 (gate/up GEMV 44 us vs 55 us with 16 KB stages; the bulk-copy ring
// delivered ~30 GB/s per SM: each stage costs a fixed ~0.5 us however small).
static bool stream_kernel_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("JSX_GEMV");
    v = (e && strcmp(e, "stream") == 0) ? 1 : 0;
  }
  return v == 1;
}

// Stage size in KB (JSX_STAGE_KB = 4, 8 or 16; default 8).  Every consumer warp
// holds one stage while it computes, so smaller stages leave more of the ring
// in flight.
static int stage_kb() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("JSX_STAGE_KB");
    const int k = e ? atoi(e) : 8;
    v = (k == 4 || k == 8 || k == 16) ? k : 8;
  }
  return v;
}

// Stage plan of the streaming kernel; false when it does not fit shared memory.
static bool make_stream_plan(const GemvArgs& a, StreamPlan* pl, size_t* smem) {
  StreamPlan p = {};
  p.stage_bytes = stage_kb() * 1024;
  p.x_bytes = (int)(((size_t)a.M * a.K * sizeof(bf16) + 15) & ~(size_t)15);
  const size_t sb = (size_t)p.stage_bytes;
  const size_t pair_bytes = (size_t)a.K * 4;  // two bf16 rows
  if (pair_bytes * 4 <= sb) p.nb = 4;
  else if (pair_bytes * 2 <= sb) p.nb = 2;
  else p.nb = 1;
  if (pair_bytes <= sb) {
    p.Kc = a.K;
    p.nchunk = 1;
  } else {
    p.Kc = (int)(sb / 4);
    p.nchunk = (a.K + p.Kc - 1) / p.Kc;
  }
  const size_t budget = 220 * 1024;  // dynamic part; the static part is < 1 KB
  const size_t fixed = (size_t)p.x_bytes + (size_t)2 * kMaxStages * sizeof(uint64_t);
  if (fixed + (size_t)kMinStages * sb > budget) return false;
  const int stages = (int)((budget - fixed) / sb);
  p.stages = stages > kMaxStages ? kMaxStages : stages;
  *smem = (size_t)p.stages * sb + (size_t)p.x_bytes + (size_t)2 * p.stages * sizeof(uint64_t);
  *pl = p;
  return true;
}

template <int M, int EPI>
static int launch_stream(const GemvArgs& a, const CommDev& c, cudaStream_t s, int max_grid,
                         const StreamPlan& pl, size_t smem) {
  auto kern = k_gemv_stream<M, EPI>;
  JSX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int grid = sm_count();
  if (grid > max_grid) grid = max_grid;
  JSX_CUDA(launch_kernel(kern, dim3(grid), dim3(kStreamThreads), smem, s, a, c, pl));
  return JSX_OK;
}

template <int EPI>
static int launch_gemv(const GemvArgs& a, const CommDev& c, cudaStream_t s, int max_grid) {
  if (stream_kernel_enabled()) {
    StreamPlan pl;
    size_t ssmem = 0;
    if (make_stream_plan(a, &pl, &ssmem)) {
      switch (a.M) {
        case 1: return launch_stream<1, EPI>(a, c, s, max_grid, pl, ssmem);
        case 2: return launch_stream<2, EPI>(a, c, s, max_grid, pl, ssmem);
        case 3: return launch_stream<3, EPI>(a, c, s, max_grid, pl, ssmem);
        case 4: return launch_stream<4, EPI>(a, c, s, max_grid, pl, ssmem);
        case 5: return launch_stream<5, EPI>(a, c, s, max_grid, pl, ssmem);
        case 6: return launch_stream<6, EPI>(a, c, s, max_grid, pl, ssmem);
        case 7: return launch_stream<7, EPI>(a, c, s, max_grid, pl, ssmem);
        case 8: return launch_stream<8, EPI>(a, c, s, max_grid, pl, ssmem);
        default: break;
      }
    }
  }
  const size_t smem = (size_t)a.M * a.K * sizeof(bf16);
  JSX_REQUIRE(smem <= kMaxDynSmem, "activations of %d x %d bf16 exceed the shared-memory stage", a.M, a.K);
  const int ngroups = a.N / kRows;
#define JSX_GEMV_CASE(MM)                                                                   \
  case MM: {                                                                                \
    auto kern = k_gemv<MM, EPI>;                                                            \
    JSX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,        \
                                  (int)smem));                                              \
    int occ = 0;                                                                            \
    JSX_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kThreads, smem));    \
    JSX_REQUIRE(occ > 0, "gemv kernel does not fit on an SM (M=%d K=%d)", a.M, a.K);       \
    int grid = sm_count() * occ;                                                            \
    const int need = (ngroups + kWarps - 1) / kWarps;                                       \
    if (grid > need) grid = need;                                                           \
    if (grid > max_grid) grid = max_grid;                                                   \
    if (grid < 1) grid = 1;                                                                 \
    JSX_CUDA(launch_kernel(kern, dim3(grid), dim3(kThreads), smem, s, a, c));              \
    return JSX_OK;                                                                          \
  }
  switch (a.M) {
    JSX_GEMV_CASE(1)
    JSX_GEMV_CASE(2)
    JSX_GEMV_CASE(3)
    JSX_GEMV_CASE(4)
    JSX_GEMV_CASE(5)
    JSX_GEMV_CASE(6)
    JSX_GEMV_CASE(7)
    JSX_GEMV_CASE(8)
    default:
      set_error("M=%d outside the decode GEMV range 1..%d", a.M, kMaxM);
      return JSX_ENOTSUP;
  }
#undef JSX_GEMV_CASE
}

static int check_common(const void* x, const void* w, int M, int K, int N) {
  JSX_REQUIRE(x && w, "null activation or weight pointer");
  JSX_REQUIRE(M >= 1 && M <= kMaxM, "M=%d outside 1..%d", M, kMaxM);
  JSX_REQUIRE(K >= 8 && K % 8 == 0, "K=%d must be a positive multiple of 8", K);
  JSX_REQUIRE(N >= kRows && N % kRows == 0, "N=%d must be a positive multiple of %d", N, kRows);
  JSX_REQUIRE(aligned16(x) && aligned16(w), "activation and weight must be 16-byte aligned");
  return JSX_OK;
}

CommDev comm_view(jsx_comm* comm);  // comm.cu

}  // namespace jsx

using namespace jsx;

extern "C" int jsx_linear(const void* x, const void* gamma, float eps, const void* w_nk,
                          const void* bias, void* y, int M, int K, int N, void* stream) {
  int st = check_common(x, w_nk, M, K, N);
  if (st) return st;
  JSX_REQUIRE(y != nullptr, "null output");
  JSX_REQUIRE(gamma == nullptr || aligned16(gamma), "gamma must be 16-byte aligned");
  GemvArgs a = {};
  a.x = (const bf16*)x; a.gamma = (const bf16*)gamma; a.eps = eps; a.w = (const bf16*)w_nk;
  a.M = M; a.K = K; a.N = N; a.bias = (const bf16*)bias; a.y = (bf16*)y;
  CommDev c = {};
  c.world = 1;
  return launch_gemv<EPI_LINEAR>(a, c, (cudaStream_t)stream, 1 << 30);
}

extern "C" int jsx_qkv_rope_cache(const void* h, const void* ln_gamma, float eps, const void* w_qkv,
                                  const void* b_qkv, const float* inv_freq,
                                  const int32_t* positions, void* q_out, void* k_cache,
                                  void* v_cache, int M, int tokens_per_seq, int K, int nq, int nkv,
                                  int head_dim, int rotary_dim, int max_seq, void* stream) {
  const int N = (nq + 2 * nkv) * head_dim;
  int st = check_common(h, w_qkv, M, K, N);
  if (st) return st;
  JSX_REQUIRE(q_out && k_cache && v_cache && positions && inv_freq, "null q/k/v/positions/inv_freq");
  JSX_REQUIRE(nq >= 1 && nkv >= 1, "bad head counts nq=%d nkv=%d", nq, nkv);
  JSX_REQUIRE(head_dim >= 2 && head_dim % 2 == 0, "head_dim=%d must be even", head_dim);
  JSX_REQUIRE(rotary_dim >= 0 && rotary_dim <= head_dim && rotary_dim % 2 == 0 &&
                  (head_dim - rotary_dim) % 2 == 0,
              "rotary_dim=%d incompatible with head_dim=%d", rotary_dim, head_dim);
  JSX_REQUIRE(tokens_per_seq >= 1 && M % tokens_per_seq == 0, "tokens_per_seq=%d must divide M=%d",
              tokens_per_seq, M);
  JSX_REQUIRE(max_seq >= 1, "max_seq=%d", max_seq);
  JSX_REQUIRE(ln_gamma == nullptr || aligned16(ln_gamma), "gamma must be 16-byte aligned");
  GemvArgs a = {};
  a.x = (const bf16*)h; a.gamma = (const bf16*)ln_gamma; a.eps = eps; a.w = (const bf16*)w_qkv;
  a.M = M; a.K = K; a.N = N; a.bias = (const bf16*)b_qkv; a.y = (bf16*)q_out;
  a.inv_freq = inv_freq; a.pos = positions; a.kc = (bf16*)k_cache; a.vc = (bf16*)v_cache;
  a.nq = nq; a.nkv = nkv; a.hd = head_dim; a.rot = rotary_dim; a.max_seq = max_seq;
  a.tps = tokens_per_seq;
  CommDev c = {};
  c.world = 1;
  return launch_gemv<EPI_QKV>(a, c, (cudaStream_t)stream, 1 << 30);
}

extern "C" int jsx_gate_up_swiglu(const void* h, const void* ln_gamma, float eps, const void* w_gu,
                                  void* act, int M, int K, int I, void* stream) {
  int st = check_common(h, w_gu, M, K, 2 * I);
  if (st) return st;
  JSX_REQUIRE(act != nullptr, "null output");
  JSX_REQUIRE(ln_gamma == nullptr || aligned16(ln_gamma), "gamma must be 16-byte aligned");
  GemvArgs a = {};
  a.x = (const bf16*)h; a.gamma = (const bf16*)ln_gamma; a.eps = eps; a.w = (const bf16*)w_gu;
  a.M = M; a.K = K; a.N = 2 * I; a.y = (bf16*)act;
  CommDev c = {};
  c.world = 1;
  return launch_gemv<EPI_SWIGLU>(a, c, (cudaStream_t)stream, 1 << 30);
}

extern "C" int jsx_row_linear_allreduce_add(jsx_comm* comm, const void* x, const void* w_nk,
                                            const void* addend, void* h, int M, int K_local, int N,
                                            void* stream) {
  int st = check_common(x, w_nk, M, K_local, N);
  if (st) return st;
  JSX_REQUIRE(h != nullptr, "null residual");
  GemvArgs a = {};
  a.x = (const bf16*)x; a.w = (const bf16*)w_nk; a.M = M; a.K = K_local; a.N = N; a.h = (bf16*)h;
  a.addend = (const bf16*)addend;
  CommDev c = {};
  c.world = 1;
  if (comm) {
    c = comm_view(comm);
    JSX_REQUIRE(c.base[0] != nullptr || c.world == 1, "comm peers not opened");
    JSX_REQUIRE(M <= c.max_tokens && N <= c.hidden,
                "M=%d N=%d exceed the comm buffer (%d tokens x %d)", M, N, c.max_tokens, c.hidden);
  }
  return launch_gemv<EPI_ROWAR>(a, c, (cudaStream_t)stream, kMaxCtas);
}

extern "C" int jsx_row_linear_allreduce(jsx_comm* comm, const void* x, const void* w_nk, void* h,
                                        int M, int K_local, int N, void* stream) {
  return jsx_row_linear_allreduce_add(comm, x, w_nk, nullptr, h, M, K_local, N, stream);
}

extern "C" int jsx_lmhead_workspace_size(int M, size_t* bytes) {
  JSX_REQUIRE(bytes && M >= 1 && M <= kMaxM, "bad arguments");
  *bytes = 256 + (size_t)kMaxM * sizeof(unsigned long long);
  return JSX_OK;
}

extern "C" int jsx_lmhead_argmax(jsx_comm* comm, const void* h, const void* norm_gamma, float eps,
                                 const void* w_vocab, int vocab_local, int vocab_offset, int M,
                                 int hidden, void* logits_out, int32_t* ids_out, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  int st = check_common(h, w_vocab, M, hidden, vocab_local);
  if (st) return st;
  size_t need = 0;
  jsx_lmhead_workspace_size(M, &need);
  JSX_REQUIRE(workspace && workspace_bytes >= need && aligned16(workspace),
              "workspace of %zu bytes (16-byte aligned) required", need);
  JSX_REQUIRE(ids_out != nullptr, "null ids_out");
  JSX_REQUIRE(vocab_offset >= 0, "vocab_offset=%d", vocab_offset);
  JSX_REQUIRE(norm_gamma == nullptr || aligned16(norm_gamma), "gamma must be 16-byte aligned");
  GemvArgs a = {};
  a.x = (const bf16*)h; a.gamma = (const bf16*)norm_gamma; a.eps = eps; a.w = (const bf16*)w_vocab;
  a.M = M; a.K = hidden; a.N = vocab_local; a.y = (bf16*)logits_out; a.vocab_offset = vocab_offset;
  a.done = (uint32_t*)workspace;
  a.keys = (unsigned long long*)((char*)workspace + 256);
  a.ids = ids_out;
  CommDev c = {};
  c.world = 1;
  if (comm) {
    c = comm_view(comm);
    JSX_REQUIRE(M <= c.max_tokens, "M=%d exceeds the comm buffer (%d tokens)", M, c.max_tokens);
  }
  return launch_gemv<EPI_LMHEAD>(a, c, (cudaStream_t)stream, 1 << 30);
}

namespace jsx {
int read_clear_step_error(uint32_t* out);  // decode_step.cu
int read_clear_tc_error(uint32_t* out);    // tc_gemm.cu
int read_clear_wide_error(uint32_t* out);  // tc_wide.cu
}

extern "C" int jsx_device_error(int* status) {
  JSX_REQUIRE(status != nullptr, "null status");
  uint32_t v = 0;
  JSX_CUDA(cudaMemcpyFromSymbol(&v, g_gemv_error, sizeof(v)));
  if (v) {
    const uint32_t zero = 0;
    JSX_CUDA(cudaMemcpyToSymbol(g_gemv_error, &zero, sizeof(zero)));
  }
  uint32_t w = 0;
  int st = jsx::read_clear_step_error(&w);
  if (st != JSX_OK) return st;
  uint32_t t = 0;
  st = jsx::read_clear_tc_error(&t);
  if (st != JSX_OK) return st;
  uint32_t u = 0;
  st = jsx::read_clear_wide_error(&u);
  if (st != JSX_OK) return st;
  *status = (v | w | t | u) ? JSX_ETIMEDOUT : JSX_OK;
  return JSX_OK;
}
