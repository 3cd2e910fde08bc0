// Whole decode step in one cooperative kernel (jsx_decode_step).
//
// A GLM-4 decode step at batch <= 8 is ~200 dependent phases (5 per layer),
// each a weight stream of 1-200 MB.  Launched as separate kernels every phase
// pays its own ramp (CTA launch, activation staging, first DRAM round trip,
// tail) — about 7 us each on B200, more than the o_proj stream itself.  Here
// one persistent grid (co-resident by cooperative launch) runs all phases:
//
//   embed | per layer: qkv -> attention -> o_proj(+AR) -> gate/up -> down(+AR) | LM head + argmax
//
// separated by grid barriers.  Before a warp waits at a barrier it issues its
// first weight batch of the next phase (weights never depend on activations),
// so the next stream is already in flight while the barrier completes.
//
// The phase bodies are the per-op kernels' device code (gemv_core.cuh,
// attn_core.cuh) with the same work split (row pair g -> CTA g mod grid), so
// results equal the per-op entry points'.  Activations written by other CTAs
// of this kernel are read through L2 (ld.global.cg).  Tensor-parallel
// all-reduces use the per-CTA flag protocol of comm.cuh with epochs
// epoch0 .. epoch0 + 2 * n_layers (the LM-head exchange takes the last).
// Every barrier and peer wait is time-bounded: a timeout sets the error word
// (jsx_device_error) and the kernel runs on to its end without waiting.
#include <stdio.h>
#include <stdlib.h>

#include "attn_core.cuh"
#include "comm.cuh"
#include "common.cuh"
#include "gemv_core.cuh"
#include "launch.cuh"

namespace jsx {

static __device__ uint32_t g_step_error;  // read and cleared through jsx_device_error

int read_clear_step_error(uint32_t* out) {
  uint32_t v = 0;
  JSX_CUDA(cudaMemcpyFromSymbol(&v, g_step_error, sizeof(v)));
  if (v) {
    const uint32_t zero = 0;
    JSX_CUDA(cudaMemcpyToSymbol(g_step_error, &zero, sizeof(zero)));
  }
  *out = v;
  return JSX_OK;
}

constexpr long long kBarrierLimitCycles = 4000000000ll;  // ~2 s at the 1965 MHz max clock

// workspace layout: [barrier 256 B][LM-head keys/done 256 B][attention workspace]
constexpr size_t kWsBarrier = 0;
constexpr size_t kWsLm = 256;
constexpr size_t kWsAttn = 512;
constexpr size_t kStepMergeSmemMax = 100 * 1024;  // two 256-thread CTAs per SM

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Grid barrier in two halves over one monotonic count bar[0] (zero when a
// launch starts).  grid_arrive: thread 0 of each CTA publishes the CTA's
// writes with a release reduction (no round trip); grid_wait: wait until the
// count reaches (barriers passed + 1) x grid.  The next phase's weight prefetch
// is issued between the halves.  grid_exit: the last CTA out of the kernel (it
// counts its exit like an arrival, after every wait of every CTA) resets the
// count for the next launch.  `gen` (barriers passed) lives in thread 0 only.
__device__ __forceinline__ void grid_arrive(uint32_t* bar, uint32_t gen) {
  __syncthreads();
  if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
}

__device__ __forceinline__ void grid_wait(uint32_t* bar, uint32_t& gen) {
  if (threadIdx.x == 0) {
    const uint32_t target = (gen + 1u) * gridDim.x;
    const long long t0 = clock64();
    uint32_t it = 0;
    while ((int)(ld_acquire_gpu(bar) - target) < 0) {
      if ((++it & 63u) == 0 && clock64() - t0 > kBarrierLimitCycles) {
        atomicOr(&g_step_error, 1u);
        break;
      }
    }
    gen = gen + 1u;
  }
  __syncthreads();
}

__device__ __forceinline__ void grid_exit(uint32_t* bar, uint32_t gen) {
  if (threadIdx.x == 0 && atomicAdd(bar, 1u) == (gen + 1u) * gridDim.x - 1u) atomicExch(bar, 0u);
}

__device__ __forceinline__ void grid_sync(uint32_t* bar, uint32_t& gen) {
  grid_arrive(bar, gen);
  grid_wait(bar, gen);
}

// Phase trace: CTA 0 stamps %globaltimer after every grid barrier (and at the end).
__device__ __forceinline__ void trace_mark(uint64_t* trace, int& n) {
  if (trace != nullptr && blockIdx.x == 0 && threadIdx.x == 0) trace[n] = globaltimer();
  ++n;
}

// First weight batch of this warp's first row pair of the next GEMV phase.
__device__ __forceinline__ void prefetch(Batch& bt, const bf16* w, int K, int N) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = blockIdx.x + gridDim.x * warp;
  const int nvec = K >> 3;
  if (g < N / kRows) load_batch(bt, reinterpret_cast<const uint4*>(w) + (size_t)g * kRows * nvec, nvec, 0, lane);
}

// The q/k/v projection with K split over warp pairs: when the row pairs are few
// (tensor parallelism >= 2) and K spans two weight batches (2048 < K <= 4096),
// warps 2j and 2j + 1 of CTA c take the two K halves of row pair c + j * grid,
// so every weight byte of the phase is in registers (prefetch_qkv_split) before
// the phase starts.  The halves are warp-reduced separately and added (first +
// second) before the epilogue.
__device__ __forceinline__ bool qkv_split_ok(int K, int N) {
  const int nvec = K >> 3, batch = 32 * kUnroll;
  return nvec > batch && nvec <= 2 * batch && N / kRows <= (kWarps / 2) * (int)gridDim.x;
}

__device__ __forceinline__ void prefetch_qkv_split(Batch& bt, const bf16* w, int K, int N) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = blockIdx.x + gridDim.x * (warp >> 1);
  const int nvec = K >> 3;
  if (g < N / kRows)
    load_batch(bt, reinterpret_cast<const uint4*>(w) + (size_t)g * kRows * nvec, nvec, (warp & 1) * 32 * kUnroll,
               lane);
}

template <int M>
__device__ __forceinline__ void gemv_qkv_split(const GemvArgs& ga, const bf16* xs, const Batch& bt) {
  __shared__ float half2[kWarps / 2][kRows][M];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = blockIdx.x + gridDim.x * (warp >> 1);
  const int nvec = ga.K >> 3;
  const bool mine = g < ga.N / kRows;
  float acc[kRows][M];
#pragma unroll
  for (int r = 0; r < kRows; ++r)
#pragma unroll
    for (int m = 0; m < M; ++m) acc[r][m] = 0.f;
  if (mine) {
    fma_batch<M>(bt, reinterpret_cast<const uint4*>(xs), nvec, (warp & 1) * 32 * kUnroll, lane, acc);
#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
      for (int m = 0; m < M; ++m) acc[r][m] = warp_sum(acc[r][m]);
    if ((warp & 1) && lane == 0) {
#pragma unroll
      for (int r = 0; r < kRows; ++r)
#pragma unroll
        for (int m = 0; m < M; ++m) half2[warp >> 1][r][m] = acc[r][m];
    }
  }
  __syncthreads();
  if (mine && !(warp & 1)) {
#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
      for (int m = 0; m < M; ++m) acc[r][m] += half2[warp >> 1][r][m];
    epi_qkv<M>(ga, g, acc, lane);
  }
}

// L2 prefetch of this warp's first row pairs of a later GEMV phase: bytes
// [from, to) of the concatenation of the groups gemv_phase will hand it
// (g = block + grid * warp + k * grid * warps); from and to are multiples of 16.
// Bulk prefetches issued by lane 0; the bytes land in L2 while this phase's
// tail, its exchange and the barrier run, so the next phase's weight reads
// start as L2 hits.
__device__ __forceinline__ void l2_prefetch_groups(const bf16* w, int K, int N, uint32_t from, uint32_t to) {
  if (to <= from || (threadIdx.x & 31) != 0) return;
  const int warp = threadIdx.x >> 5, G = gridDim.x, ngroups = N / kRows;
  const uint32_t pair = (uint32_t)kRows * (uint32_t)K * 2u;  // K % 8 == 0: a multiple of 16
  uint32_t at = 0;  // byte offset of group g in the warp's concatenation
  for (int g = blockIdx.x + G * warp; g < ngroups && at < to; g += G * kWarps, at += pair) {
    const uint32_t lo = from > at ? from - at : 0u;
    const uint32_t hi = to - at < pair ? to - at : pair;
    if (hi <= lo) continue;
    const char* p = reinterpret_cast<const char*>(w) + (size_t)g * pair + lo;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(hi - lo) : "memory");
  }
}

// L2 prefetch of a small vector that a later phase reads once per step (norm
// weights, the q/k/v bias): one bulk request from thread 0 of CTA `cta`, so the
// later phase's first read of it is an L2 hit rather than an HBM round trip on
// its critical path.  Skipped for a pointer that is not 16-byte aligned.
__device__ __forceinline__ void l2_prefetch_vec(const void* p, uint32_t bytes, int cta) {
  if (p == nullptr || bytes < 16u || (reinterpret_cast<uintptr_t>(p) & 15u) != 0 || (int)blockIdx.x != cta ||
      threadIdx.x != 0)
    return;
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes & ~15u) : "memory");
}

// Latest %globaltimer of any CTA at this point (trace of the exchange phases).
__device__ __forceinline__ void trace_max(uint64_t* slot) {
  if (slot == nullptr) return;
  __syncthreads();
  if (threadIdx.x == 0) atomicMax(reinterpret_cast<unsigned long long*>(slot), (unsigned long long)globaltimer());
}

// Consumer-side split merge (stage_attn_merge): enabled when the records of all
// groups are small (few groups: tensor parallelism >= 4 at GLM-4 shapes), so every
// o_proj CTA can read them all; its shared weights hold groups x splits x gi floats.
constexpr int kMergeWeights = 1024;
constexpr size_t kMergeRecordBytes = 80 * 1024;

// One GEMV phase (bt holds the first batch of this warp's first group).
template <int M, int EPI>
__device__ __forceinline__ void gemv_phase(const GemvArgs& ga, const CommDev& c, bool multi, uint32_t epoch,
                                           const bf16* xs, Batch& bt, unsigned long long (&best)[M]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nvec = ga.K >> 3, ngroups = ga.N / kRows, G = gridDim.x;
  const uint4* wbase = reinterpret_cast<const uint4*>(ga.w);
  const size_t gvecs = (size_t)kRows * nvec;
  const uint4* xv = reinterpret_cast<const uint4*>(xs);
  for (int g = blockIdx.x + G * warp; g < ngroups; g += G * kWarps) {
    const uint4* wv = wbase + (size_t)g * gvecs;
    float acc[kRows][M];
#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
      for (int m = 0; m < M; ++m) acc[r][m] = 0.f;
    for (int base = 0; base < nvec; base += 32 * kUnroll) {
      if (base > 0) load_batch(bt, wv, nvec, base, lane);
      fma_batch<M>(bt, xv, nvec, base, lane, acc);
    }
    const int gn = g + G * kWarps;
    if (gn < ngroups) load_batch(bt, wbase + (size_t)gn * gvecs, nvec, 0, lane);
#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
      for (int m = 0; m < M; ++m) acc[r][m] = warp_sum(acc[r][m]);

    if constexpr (EPI == EPI_QKV) {
      epi_qkv<M>(ga, g, acc, lane);
    } else if constexpr (EPI == EPI_SWIGLU) {
      epi_swiglu<M>(ga, g, acc, lane);
    } else if constexpr (EPI == EPI_ROWAR) {
      if (lane < kRows * M) {
        const int r = lane / M, m = lane - (lane / M) * M;
        const int row = g * kRows + r;
        const float v = pick<M>(acc, r, m);
        if (!multi) {
          bf16* hp = ga.h + (size_t)m * ga.N + row;
          *hp = __float2bfloat16_rn(__bfloat162float(__ldcg(hp)) + rbf(v));
        } else {
          for (int d = 0; d < c.world; ++d) ll_put(data_ptr(c, d, epoch & 1, c.rank, m) + row, v, epoch);
        }
      }
    } else if constexpr (EPI == EPI_LMHEAD) {
      unsigned long long key = 0ull;
      int mine = -1;
      if (lane < kRows * M) {
        const int r = lane / M, m = lane - (lane / M) * M;
        const int row = g * kRows + r;
        const float v = rbf(pick<M>(acc, r, m));
        if (ga.y) ga.y[(size_t)m * ga.N + row] = __float2bfloat16_rn(v);
        key = argmax_key(v, (uint32_t)(ga.vocab_offset + row));
        mine = m;
      }
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const unsigned long long k = warp_max_u64(mine == m ? key : 0ull);
        best[m] = k > best[m] ? k : best[m];
      }
    }
  }
}

// Row-parallel exchange of one all-reduce phase: the rows this CTA computed,
// read from every rank's LL slots once they carry the phase's epoch, summed in
// rank order and added to the residual.  The residual and every rank's slot of
// an entry are loaded before any is waited on (one round trip when the peers'
// pushes have landed); a slot whose epoch is not there yet is then polled.
__device__ __forceinline__ unsigned long long ll_load(const unsigned long long* slot) {
  unsigned long long w;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(slot) : "memory");
  return w;
}

// Out of line: the loop-invariant addressing of the exchange is not hoisted
// into the GEMV loops, where registers are scarce.  `slots` = this rank's LL
// words of the phase's parity, [src][max_tokens][n] u64.
template <int M>
__device__ __noinline__ void allreduce_rows_impl(bf16* h, int n, const unsigned long long* slots, size_t sstride,
                                                 int world, int max_tokens, uint32_t* state,
                                                 unsigned long long timeout_ns, uint32_t epoch) {
  const int ngroups = n / kRows, G = gridDim.x;
  const int my_groups = (ngroups - (int)blockIdx.x + G - 1) / G;
  const int entries = my_groups * kRows * M;
  for (int e = threadIdx.x; e < entries; e += blockDim.x) {
    const int gl = e / (kRows * M);
    const int rem = e - gl * kRows * M;
    const int r = rem / M, m = rem - (rem / M) * M;
    const int row = (blockIdx.x + G * gl) * kRows + r;
    bf16* hp = h + (size_t)m * n + row;
    const float h0 = __bfloat162float(__ldcg(hp));
    // slot of source src: p0 + src * sstride; every source's slot is loaded
    // before any is checked
    const unsigned long long* p0 = slots + (size_t)m * n + row;
    unsigned long long w[kMaxRanks];
#pragma unroll
    for (int src = 0; src < kMaxRanks; ++src)
      if (src < world) w[src] = ll_load(p0 + src * sstride);
    float s = 0.f;
    bool all = true;
#pragma unroll
    for (int src = 0; src < kMaxRanks; ++src) {
      if (src < world) {
        all = all && (uint32_t)(w[src] >> 32) == epoch;
        s += __uint_as_float((uint32_t)w[src]);
      }
    }
    if (!all) {
      // some push has not landed yet: reload every slot still without the
      // epoch, all in flight together (one round trip per pass), until all
      // carry it; bounded by the comm timeout and the error word
      const uint64_t t0 = globaltimer();
#pragma unroll 1
      for (uint32_t it = 1; !all; ++it) {
#pragma unroll
        for (int src = 0; src < kMaxRanks; ++src)
          if (src < world && (uint32_t)(w[src] >> 32) != epoch) w[src] = ll_load(p0 + src * sstride);
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
      s = 0.f;
#pragma unroll
      for (int src = 0; src < kMaxRanks; ++src)
        if (src < world) s += (uint32_t)(w[src] >> 32) == epoch ? __uint_as_float((uint32_t)w[src]) : 0.f;
    }
    *hp = __float2bfloat16_rn(h0 + rbf(s));
  }
}

template <int M>
__device__ __forceinline__ void allreduce_rows(const GemvArgs& ga, const CommDev& c, uint32_t epoch) {
  allreduce_rows_impl<M>(ga.h, ga.N, data_ptr(c, c.rank, epoch & 1, 0, 0), (size_t)c.max_tokens * c.hidden,
                         c.world, c.max_tokens, c.state, c.timeout_ns, epoch);
}

// o_proj staging with the attention's split merge folded in (small groups,
// at.no_merge): every CTA combines the split records of every (sequence, head
// group) itself, after the grid barrier that follows the attention, instead of
// the last split of each group merging them (an atomic round trip and a merge
// on the attention's critical path).  The arithmetic is attn_finish's, in the
// same order (bit-identical): per head M = max_t m_t, e_t = exp(m_t - M),
// L = warp sum of l_t e_t, w_t = e_t / L, out = sum_t fma(acc_t, w_t) -> bf16.
// cw: shared weights, groups x splits x gi floats.
template <int M>
__device__ __forceinline__ void stage_attn_merge(const AttnArgs& at, bf16* xs, float* cw) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gi = at.gi, hd = at.hd, stride = split_stride(gi, hd);
  const int G = at.nq / at.nkv, groups = M * at.nkv * at.hg, qd = at.nq * hd;
  for (int pr = warp; pr < groups * gi; pr += kWarps) {
    const int vb = pr / gi, h = pr - vb * gi;
    const int b = vb / (at.nkv * at.hg);
    int cur = at.pos[b];
    if (cur > at.max_seq - 1) cur = at.max_seq - 1;
    if (cur < 0) cur = 0;
    const int used = (cur + kChunk) / kChunk;
    const float* pb = at.part + (size_t)vb * at.splits * stride;
    float Mx = -INFINITY;
    for (int t = lane; t < used; t += 32) Mx = fmaxf(Mx, __ldcg(pb + (size_t)t * stride + gi * hd + h));
    Mx = warp_max(Mx);
    float L = 0.f;
    float* w = cw + (size_t)vb * at.splits * gi;
    for (int t = lane; t < used; t += 32) {
      const float e = expf(__ldcg(pb + (size_t)t * stride + gi * hd + h) - Mx);
      w[t * gi + h] = e;
      L = fmaf(__ldcg(pb + (size_t)t * stride + gi * hd + gi + h), e, L);
    }
    L = warp_sum(L);
    for (int t = lane; t < used; t += 32) w[t * gi + h] = w[t * gi + h] / L;
  }
  __syncthreads();
  const int per = (gi * hd) >> 1;  // float2 outputs per group
  for (int i = tid; i < groups * per; i += kThreads) {
    const int vb = i / per, k = i - vb * per;
    const int b = vb / (at.nkv * at.hg), kvh = (vb / at.hg) % at.nkv, j = vb % at.hg;
    const int h = (k << 1) / hd;
    int cur = at.pos[b];
    if (cur > at.max_seq - 1) cur = at.max_seq - 1;
    if (cur < 0) cur = 0;
    const int used = (cur + kChunk) / kChunk;
    const float2* r2 = reinterpret_cast<const float2*>(at.part + (size_t)vb * at.splits * stride);
    const float* w = cw + (size_t)vb * at.splits * gi;
    float2 o = make_float2(0.f, 0.f);
    // eight splits' loads in flight before their products (the same t order)
    for (int t0 = 0; t0 < used; t0 += 8) {
      float2 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        v[u] = t0 + u < used ? __ldcg(r2 + (size_t)(t0 + u) * (stride >> 1) + k) : make_float2(0.f, 0.f);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (t0 + u < used) {
          const float wt = w[(t0 + u) * gi + h];
          o.x = fmaf(v[u].x, wt, o.x);
          o.y = fmaf(v[u].y, wt, o.y);
        }
      }
    }
    const int col = (kvh * G + j * gi) * hd + (k << 1);
    *reinterpret_cast<uint32_t*>(xs + (size_t)b * qd + col) = pack2(o.x, o.y);
  }
  __syncthreads();
}

// opts: kOptConsumerMerge, kOptDistMerge (host-selected variants; same results)
constexpr int kOptConsumerMerge = 1;  // the o_proj staging merges the attention splits
constexpr int kOptDistMerge = 2;      // every split of a group merges a share of its heads

template <int M>
__global__ void __launch_bounds__(kThreads, 2) k_decode_step(jsx_decode_step_args a, CommDev c, int opts) {
  const int cmerge = opts & kOptConsumerMerge;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ float cmerge_w[kMergeWeights];
  bf16* xs = reinterpret_cast<bf16*>(smem_raw);
  __shared__ bool is_last;
  __shared__ unsigned long long cta_best[kWarps][M];
  __shared__ unsigned long long fin[M];

  unsigned char* ws = reinterpret_cast<unsigned char*>(a.workspace);
  uint32_t* bar = reinterpret_cast<uint32_t*>(ws + kWsBarrier);
  uint32_t* lm_done = reinterpret_cast<uint32_t*>(ws + kWsLm);
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(ws + kWsLm + 64);
  const jsx_layer_weights* layers = a.layers;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool multi = c.world > 1;
  int tn = 0;
  uint32_t gen = 0;
  const uint32_t epoch0 = multi ? read_epoch(c) : 0u;
  const int qdim = a.n_heads * a.head_dim;
  const int qkv_rows = (a.n_heads + 2 * a.n_kv_heads) * a.head_dim;

  // ---- embedding (layers/embedding.py:35-51), CTA 0 ----
  if (blockIdx.x == 0) {
    const int hv = a.hidden >> 3;
    for (int i = threadIdx.x; i < M * hv; i += blockDim.x) {
      const int m = i / hv, v = i - (i / hv) * hv;
      const int id = a.ids[m];
      uint4 val;
      if (id < 0 || id >= a.vocab) {
        const uint32_t nan2 = 0x7fc07fc0u;
        val = make_uint4(nan2, nan2, nan2, nan2);
      } else {
        val = reinterpret_cast<const uint4*>(a.embed)[(size_t)id * hv + v];
      }
      reinterpret_cast<uint4*>(a.h)[(size_t)m * hv + v] = val;
    }
  }
  Batch bt;
  unsigned long long best[M];
#pragma unroll
  for (int m = 0; m < M; ++m) best[m] = 0ull;
  const bool qkv_split = qkv_split_ok(a.hidden, qkv_rows);
  grid_arrive(bar, gen);
  if (qkv_split) prefetch_qkv_split(bt, reinterpret_cast<const bf16*>(layers[0].w_qkv), a.hidden, qkv_rows);
  else prefetch(bt, reinterpret_cast<const bf16*>(layers[0].w_qkv), a.hidden, qkv_rows);
  l2_prefetch_vec(layers[0].ln1, 2u * a.hidden, 0);
  l2_prefetch_vec(layers[0].b_qkv, 2u * qkv_rows, 1);
  grid_wait(bar, gen);
  trace_mark(a.trace, tn);

  AttnArgs at;
  at.q = reinterpret_cast<const bf16*>(a.q);
  at.out = reinterpret_cast<bf16*>(a.attn);
  at.pos = a.positions;
  at.B = M;
  at.nq = a.n_heads;
  at.nkv = a.n_kv_heads;
  at.hd = a.head_dim;
  at.max_seq = a.max_seq;
  const AttnLayout lay = attn_layout(M, a.n_heads, a.n_kv_heads, a.head_dim, a.max_seq);
  at.splits = lay.splits;
  at.gi = lay.gi;
  at.hg = lay.hg;
  at.no_merge = cmerge;
  at.scale = a.scale;
  at.cnt = reinterpret_cast<uint32_t*>(ws + kWsAttn + 256);
  at.part = reinterpret_cast<float*>(ws + kWsAttn + lay.counter_bytes);
  const int attn_items = M * a.n_kv_heads * lay.hg * lay.splits;
  // distributed split merge: every item on its own CTA (all co-resident: the
  // split CTAs of a group wait for one another), the tensor-core item (its
  // shared memory holds the merge's weights and kSeg staged accumulators)
  at.dist_err = (!cmerge && (opts & kOptDistMerge) && attn_items <= (int)gridDim.x &&
                 attn_use_mma(lay.gi, a.head_dim) && lay.splits <= 2048)
                    ? &g_step_error
                    : nullptr;
  const bool attn_pre = attn_use_mma(lay.gi, a.head_dim) && (int)blockIdx.x < attn_items;

  for (int l = 0; l < a.n_layers; ++l) {
    const jsx_layer_weights L = layers[l];
    uint64_t* tp = a.trace_phase ? a.trace_phase + 15 * l : nullptr;  // [phase][point]
#define JSX_TP(ph, pt) trace_max(tp ? tp + 3 * (ph) + (pt) : nullptr)
    // ---- q/k/v + bias + RoPE + KV write (models/glm4.py:118-120) ----
    {
      GemvArgs ga = {};
      ga.x = reinterpret_cast<const bf16*>(a.h);
      ga.gamma = reinterpret_cast<const bf16*>(L.ln1);
      ga.eps = a.eps;
      ga.w = reinterpret_cast<const bf16*>(L.w_qkv);
      ga.M = M; ga.K = a.hidden; ga.N = qkv_rows;
      ga.bias = reinterpret_cast<const bf16*>(L.b_qkv);
      ga.y = reinterpret_cast<bf16*>(a.q);
      ga.inv_freq = a.inv_freq; ga.pos = a.positions;
      ga.kc = reinterpret_cast<bf16*>(L.k_cache); ga.vc = reinterpret_cast<bf16*>(L.v_cache);
      ga.nq = a.n_heads; ga.nkv = a.n_kv_heads; ga.hd = a.head_dim; ga.rot = a.rotary_dim;
      ga.max_seq = a.max_seq; ga.tps = 1;
      stage_x<M, false, true>(ga, xs);
      JSX_TP(0, 0);
      if (qkv_split) gemv_qkv_split<M>(ga, xs, bt);
      else gemv_phase<M, EPI_QKV>(ga, c, multi, 0u, xs, bt, best);
      JSX_TP(0, 1);
      l2_prefetch_groups(reinterpret_cast<const bf16*>(L.w_o), qdim, a.hidden, 0u, a.l2_next_bytes);
      JSX_TP(0, 2);
    }
    at.trace = a.trace ? a.trace + (2 + 5 * a.n_layers) + 8 * l : nullptr;
    at.kc = reinterpret_cast<const bf16*>(L.k_cache);
    at.vc = reinterpret_cast<const bf16*>(L.v_cache);
    grid_arrive(bar, gen);
    // the cache rows of this CTA's first attention item that earlier steps
    // wrote are staged while the barrier completes
    int pre_cur = 0;
    if (attn_pre) pre_cur = attn_prefetch_mma<kThreads>(at, blockIdx.x % at.splits, blockIdx.x / at.splits, smem_raw);
    grid_wait(bar, gen);
  trace_mark(a.trace, tn);
    // ---- attention over cache rows [0, pos] (layers/attention.py:148-153) ----
    // HBM is idle while the attention's short dependency chain runs: gate/up rows go to L2
    l2_prefetch_groups(reinterpret_cast<const bf16*>(L.w_gu), a.hidden, 2 * a.inter, 0u, a.l2_attn_bytes);
    JSX_TP(1, 0);
    for (int it = blockIdx.x; it < attn_items; it += gridDim.x) {
      if (attn_pre && it == (int)blockIdx.x)
        attn_item_mma<kThreads, true, true, true>(at, it % at.splits, it / at.splits, smem_raw, pre_cur);
      else
        attn_item_any<kThreads, true, true>(at, it % at.splits, it / at.splits, smem_raw);
    }
    JSX_TP(1, 1);
    JSX_TP(1, 2);
    grid_arrive(bar, gen);
    prefetch(bt, reinterpret_cast<const bf16*>(L.w_o), qdim, a.hidden);
    l2_prefetch_vec(L.ln2, 2u * a.hidden, (int)gridDim.x - 1);
    grid_wait(bar, gen);
  trace_mark(a.trace, tn);
    // ---- o_proj + all-reduce + residual (layers/attention.py:159, models/glm4.py:124) ----
    {
      GemvArgs ga = {};
      ga.x = reinterpret_cast<const bf16*>(a.attn);
      ga.w = reinterpret_cast<const bf16*>(L.w_o);
      ga.M = M; ga.K = qdim; ga.N = a.hidden;
      ga.h = reinterpret_cast<bf16*>(a.h);
      const uint32_t ep = epoch0 + 2u * l;
      if (cmerge) stage_attn_merge<M>(at, xs, cmerge_w);
      else stage_x<M, false, true>(ga, xs);
      JSX_TP(2, 0);
      gemv_phase<M, EPI_ROWAR>(ga, c, multi, ep, xs, bt, best);
      uint64_t* ar = a.trace_ar ? a.trace_ar + 4 * l : nullptr;
      trace_max(ar);
      JSX_TP(2, 1);
      l2_prefetch_groups(reinterpret_cast<const bf16*>(L.w_gu), a.hidden, 2 * a.inter, a.l2_attn_bytes,
                         a.l2_next_bytes);
      if (multi) allreduce_rows<M>(ga, c, ep);
      trace_max(ar ? ar + 1 : nullptr);
      JSX_TP(2, 2);
    }
    grid_arrive(bar, gen);
    prefetch(bt, reinterpret_cast<const bf16*>(L.w_gu), a.hidden, 2 * a.inter);
    grid_wait(bar, gen);
  trace_mark(a.trace, tn);
    // ---- post-attention norm + gate/up + SwiGLU (models/glm4.py:128, :46-48) ----
    {
      GemvArgs ga = {};
      ga.x = reinterpret_cast<const bf16*>(a.h);
      ga.gamma = reinterpret_cast<const bf16*>(L.ln2);
      ga.eps = a.eps;
      ga.w = reinterpret_cast<const bf16*>(L.w_gu);
      ga.M = M; ga.K = a.hidden; ga.N = 2 * a.inter;
      ga.y = reinterpret_cast<bf16*>(a.act);
      stage_x<M, false, true>(ga, xs);
      JSX_TP(3, 0);
      gemv_phase<M, EPI_SWIGLU>(ga, c, multi, 0u, xs, bt, best);
      JSX_TP(3, 1);
      l2_prefetch_groups(reinterpret_cast<const bf16*>(L.w_d), a.inter, a.hidden, 0u, a.l2_next_bytes);
      JSX_TP(3, 2);
    }
    grid_arrive(bar, gen);
    prefetch(bt, reinterpret_cast<const bf16*>(L.w_d), a.inter, a.hidden);
    if (l + 1 < a.n_layers) {
      l2_prefetch_vec(layers[l + 1].ln1, 2u * a.hidden, (int)gridDim.x - 1);
      l2_prefetch_vec(layers[l + 1].b_qkv, 2u * qkv_rows, (int)gridDim.x - 2);
    } else if (a.head) {
      l2_prefetch_vec(a.final_norm, 2u * a.hidden, (int)gridDim.x - 1);
    }
    grid_wait(bar, gen);
  trace_mark(a.trace, tn);
    // ---- down_proj + all-reduce + residual (models/glm4.py:49, :130) ----
    {
      GemvArgs ga = {};
      ga.x = reinterpret_cast<const bf16*>(a.act);
      ga.w = reinterpret_cast<const bf16*>(L.w_d);
      ga.M = M; ga.K = a.inter; ga.N = a.hidden;
      ga.h = reinterpret_cast<bf16*>(a.h);
      const uint32_t ep = epoch0 + 2u * l + 1u;
      stage_x<M, false, true>(ga, xs);
      JSX_TP(4, 0);
      gemv_phase<M, EPI_ROWAR>(ga, c, multi, ep, xs, bt, best);
      uint64_t* ar = a.trace_ar ? a.trace_ar + 4 * l + 2 : nullptr;
      trace_max(ar);
      JSX_TP(4, 1);
      if (l + 1 < a.n_layers)
        l2_prefetch_groups(reinterpret_cast<const bf16*>(layers[l + 1].w_qkv), a.hidden, qkv_rows, 0u,
                           a.l2_next_bytes);
      else if (a.head)
        l2_prefetch_groups(reinterpret_cast<const bf16*>(a.lm_head), a.hidden, a.vocab_local, 0u,
                           a.l2_next_bytes);
      if (multi) allreduce_rows<M>(ga, c, ep);
      trace_max(ar ? ar + 1 : nullptr);
      JSX_TP(4, 2);
    }
#undef JSX_TP
    grid_arrive(bar, gen);
    if (l + 1 < a.n_layers && qkv_split)
      prefetch_qkv_split(bt, reinterpret_cast<const bf16*>(layers[l + 1].w_qkv), a.hidden, qkv_rows);
    else if (l + 1 < a.n_layers)
      prefetch(bt, reinterpret_cast<const bf16*>(layers[l + 1].w_qkv), a.hidden, qkv_rows);
    else if (a.head)
      prefetch(bt, reinterpret_cast<const bf16*>(a.lm_head), a.hidden, a.vocab_local);
    grid_wait(bar, gen);
  trace_mark(a.trace, tn);
  }

  const uint32_t last_epoch = epoch0 + 2u * a.n_layers - 1u;
  if (!a.head) {
    // prefill step: no LM head; advance the positions once every CTA is done
    if (blockIdx.x == 0 && threadIdx.x < M) {
      if (threadIdx.x == 0 && a.trace) a.trace[tn] = globaltimer();
      if (a.advance) a.positions[threadIdx.x] += 1;
      if (threadIdx.x == 0 && multi) c.state[kCalls] = last_epoch;
    }
    grid_exit(bar, gen);
    return;
  }

  // ---- final norm + LM head + greedy argmax (models/glm4.py:193, :251; runner.py:297) ----
  {
    GemvArgs ga = {};
    ga.x = reinterpret_cast<const bf16*>(a.h);
    ga.gamma = reinterpret_cast<const bf16*>(a.final_norm);
    ga.eps = a.eps;
    ga.w = reinterpret_cast<const bf16*>(a.lm_head);
    ga.M = M; ga.K = a.hidden; ga.N = a.vocab_local;
    ga.y = reinterpret_cast<bf16*>(a.logits);
    ga.vocab_offset = a.vocab_offset;
    stage_x<M, false, true>(ga, xs);
    gemv_phase<M, EPI_LMHEAD>(ga, c, multi, 0u, xs, bt, best);
  }
  if (lane == 0) {
#pragma unroll
    for (int m = 0; m < M; ++m) cta_best[warp][m] = best[m];
  }
  __syncthreads();
  if (threadIdx.x < M) {
    unsigned long long b = 0ull;
    for (int w = 0; w < kWarps; ++w) b = cta_best[w][threadIdx.x] > b ? cta_best[w][threadIdx.x] : b;
    atomicMax(keys + threadIdx.x, b);
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) is_last = atomicAdd(lm_done, 1u) == gridDim.x - 1;
  __syncthreads();
  grid_exit(bar, gen);
  if (!is_last) return;
  __threadfence();
  if (threadIdx.x < M) fin[threadIdx.x] = atomicAdd(keys + threadIdx.x, 0ull);
  __syncthreads();
  if (multi) {
    const uint32_t ep = last_epoch + 1u;
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
    keys[threadIdx.x] = 0ull;
    if (a.advance) a.positions[threadIdx.x] += 1;
  }
  if (threadIdx.x == 0) {
    *lm_done = 0u;
    if (a.trace) a.trace[tn] = globaltimer();
  }
}

static size_t step_smem(const jsx_decode_step_args& a) {
  const int M = a.batch;
  int kmax = a.hidden;
  if (a.inter > kmax) kmax = a.inter;
  if (a.n_heads * a.head_dim > kmax) kmax = a.n_heads * a.head_dim;
  const size_t x = (size_t)M * kmax * sizeof(bf16);
  const AttnLayout lay = attn_layout(M, a.n_heads, a.n_kv_heads, a.head_dim, a.max_seq);
  size_t at = attn_smem(lay.gi, a.head_dim, lay.splits);
  if (attn_use_mma(lay.gi, a.head_dim)) {
    // room for the split merge to take every record into shared memory at once
    // (attn_finish), while two CTAs still fit on an SM
    const size_t merge = (size_t)kMmaHeads * kRowPad * 2 + (size_t)lay.splits * (lay.stride + lay.gi) * 4;
    if (merge > at && merge <= kStepMergeSmemMax) at = merge;
  }
  return x > at ? x : at;
}

// Whether the o_proj staging merges the attention splits (stage_attn_merge):
// only when JSX_STEP_CMERGE=1 and every group's records together fit
// kMergeWeights weights and kMergeRecordBytes bytes.  Off by default: at GLM-4
// shapes, tensor parallelism 4, context 1024 it takes the attention phase from
// 7.9 to 4.1 us but o_proj from 8.8 to 15.8 us (every o_proj CTA reads all
// 66 KB of records), 536 -> 495 tokens/s.
static int consumer_merge(const jsx_decode_step_args& a) {
  const AttnLayout lay = attn_layout(a.batch, a.n_heads, a.n_kv_heads, a.head_dim, a.max_seq);
  const size_t groups = (size_t)a.batch * a.n_kv_heads * lay.hg;
  const bool fits = groups * lay.splits * lay.gi <= (size_t)kMergeWeights &&
                    groups * lay.splits * lay.stride * sizeof(float) <= kMergeRecordBytes;
  const char* env = getenv("JSX_STEP_CMERGE");
  return (env != nullptr && atoi(env) != 0 && fits) ? 1 : 0;
}

static size_t step_workspace(const jsx_decode_step_args& a) {
  return kWsAttn + attn_layout(a.batch, a.n_heads, a.n_kv_heads, a.head_dim, a.max_seq).bytes;
}

static int check_step(const jsx_decode_step_args* a) {
  JSX_REQUIRE(a != nullptr, "null args");
  JSX_REQUIRE(a->batch >= 1 && a->batch <= kMaxM, "batch=%d outside 1..%d", a->batch, kMaxM);
  JSX_REQUIRE(a->hidden >= 8 && a->hidden % 8 == 0, "hidden=%d must be a multiple of 8", a->hidden);
  JSX_REQUIRE(a->n_heads >= 1 && a->n_kv_heads >= 1 && a->n_heads % a->n_kv_heads == 0,
              "heads %d / kv heads %d", a->n_heads, a->n_kv_heads);
  JSX_REQUIRE(a->head_dim >= 8 && a->head_dim % 8 == 0, "head_dim=%d must be a multiple of 8", a->head_dim);
  JSX_REQUIRE(a->rotary_dim >= 0 && a->rotary_dim <= a->head_dim && a->rotary_dim % 2 == 0,
              "rotary_dim=%d", a->rotary_dim);
  JSX_REQUIRE(a->inter >= 8 && a->inter % 8 == 0, "inter=%d must be a multiple of 8", a->inter);
  JSX_REQUIRE(a->vocab_local >= 2 && a->vocab_local % 2 == 0 && a->vocab >= a->vocab_local,
              "vocab_local=%d", a->vocab_local);
  JSX_REQUIRE(a->max_seq >= 1 && a->n_layers >= 1, "max_seq=%d n_layers=%d", a->max_seq, a->n_layers);
  JSX_REQUIRE(a->layers && a->embed && a->final_norm && a->lm_head && a->inv_freq && a->ids &&
                  a->positions && a->h && a->q && a->attn && a->act && a->workspace,
              "null pointer argument");
  JSX_REQUIRE(aligned16(a->embed) && aligned16(a->lm_head) && aligned16(a->final_norm) && aligned16(a->h) &&
                  aligned16(a->q) && aligned16(a->attn) && aligned16(a->act) && aligned16(a->workspace),
              "tensors must be 16-byte aligned");
  JSX_REQUIRE(a->workspace_bytes >= step_workspace(*a), "workspace of %zu bytes required",
              step_workspace(*a));
  JSX_REQUIRE(a->l2_next_bytes % 16 == 0 && a->l2_attn_bytes % 16 == 0,
              "L2 prefetch sizes %u / %u must be multiples of 16", a->l2_next_bytes, a->l2_attn_bytes);
  return JSX_OK;
}

}  // namespace jsx

using namespace jsx;


extern "C" int jsx_decode_step_workspace_size(const jsx_decode_step_args* args, size_t* bytes) {
  JSX_REQUIRE(args && bytes, "null argument");
  JSX_REQUIRE(args->batch >= 1 && args->n_kv_heads >= 1 && args->n_heads % args->n_kv_heads == 0 &&
                  args->max_seq >= 1,
              "bad shape");
  *bytes = step_workspace(*args);
  return JSX_OK;
}

namespace jsx {
CommDev comm_view(jsx_comm* comm);  // comm.cu
}

extern "C" int jsx_decode_step(jsx_comm* comm, const jsx_decode_step_args* args, void* stream) {
  int st = check_step(args);
  if (st) return st;
  const jsx_decode_step_args& a = *args;
  CommDev c = {};
  c.world = 1;
  if (comm) {
    c = jsx::comm_view(comm);
    JSX_REQUIRE(a.batch <= c.max_tokens && a.hidden <= c.hidden,
                "batch %d / hidden %d exceed the comm buffer", a.batch, a.hidden);
  }
  const size_t smem = step_smem(a);
  JSX_REQUIRE(smem <= kMaxDynSmem, "step needs %zu bytes of shared memory", smem);
  // JSX_STEP_DMERGE=1: every split of an attention group merges a share of its
  // heads after a bounded wait for the others, instead of the last split
  // merging them all (the per-op kernel's form).  Off by default: at GLM-4
  // shapes, context 1024, the two were within 0.3 % of each other at tensor
  // parallelism 1 and 4.
  const char* dm = getenv("JSX_STEP_DMERGE");
  const int opts = (consumer_merge(a) ? kOptConsumerMerge : 0) | ((dm && atoi(dm) != 0) ? kOptDistMerge : 0);
#define JSX_STEP_CASE(MM)                                                                    \
  case MM: {                                                                                 \
    auto kern = k_decode_step<MM>;                                                           \
    JSX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,         \
                                  (int)smem));                                               \
    int occ = 0;                                                                             \
    JSX_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kThreads, smem));     \
    JSX_REQUIRE(occ > 0, "decode step kernel does not fit on an SM");                       \
    if (occ > 2) occ = 2;                                                                    \
    int grid = sm_count() * occ;                                                             \
    if (grid > kMaxCtas) grid = kMaxCtas;                                                    \
    cudaLaunchConfig_t cfg = {};                                                             \
    cfg.gridDim = dim3(grid);                                                                \
    cfg.blockDim = dim3(kThreads);                                                           \
    cfg.dynamicSmemBytes = smem;                                                             \
    cfg.stream = (cudaStream_t)stream;                                                       \
    cudaLaunchAttribute attr[1];                                                             \
    attr[0].id = cudaLaunchAttributeCooperative;                                             \
    attr[0].val.cooperative = 1;                                                             \
    cfg.attrs = attr;                                                                        \
    cfg.numAttrs = 1;                                                                        \
    JSX_CUDA(cudaLaunchKernelEx(&cfg, kern, a, c, opts));                                    \
    return JSX_OK;                                                                           \
  }
  switch (a.batch) {
    JSX_STEP_CASE(1)
    JSX_STEP_CASE(2)
    JSX_STEP_CASE(3)
    JSX_STEP_CASE(4)
    JSX_STEP_CASE(5)
    JSX_STEP_CASE(6)
    JSX_STEP_CASE(7)
    JSX_STEP_CASE(8)
    default:
      break;
  }
#undef JSX_STEP_CASE
  set_error("batch %d outside the decode-step kernel set", a.batch);
  return JSX_ENOTSUP;
}
