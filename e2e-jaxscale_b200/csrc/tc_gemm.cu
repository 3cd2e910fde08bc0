// Tensor-core decode projections for 1..32 tokens (batch > 8): tcgen05 + TMA.
//
// At batch 32 a weight element feeds 64 flops; the CUDA-core GEMV would be
// compute bound (~8x the HBM time), so these projections run on the 5th-gen
// tensor cores.  Shapes are "skinny": D[128 weight rows, 32 tokens] per tile,
// the weight tile is the MMA's A operand (M = 128) and the token activations
// the B operand (N = 32, zero-filled by TMA beyond the real token count), both
// K-major bf16 with the 128-byte swizzle, fp32 accumulation in TMEM.
//
// Work split.  A tile of 128 weight rows is computed by one thread-block
// cluster of S CTAs (S = 1..8); CTA r of the cluster takes the r-th slice of
// K.  Clusters are persistent: cluster c handles tiles c, c + #clusters, ...
// Inside a CTA the warps specialise:
//   warp 0 / lane 0   TMA producer: the A (16 KB) and B (4 KB) boxes of each
//                     64-wide K block into an 8-stage ring, running ahead
//                     across tiles;
//   warp 1 / lane 0   MMA issuer: 4 tcgen05.mma (K = 16) per stage into one of
//                     two TMEM accumulators (double buffer, 2 x 32 columns);
//                     tcgen05.commit hands stages and accumulators back;
//   warps 2..5        epilogue: tcgen05.ld 32x32b.x32 (thread = one weight row
//                     x 32 tokens) into a shared-memory exchange buffer; the
//                     S partial tiles of the cluster are then read through
//                     distributed shared memory and summed in rank order by
//                     the CTA that owns the rows (CTA r finishes row pairs
//                     [64 r / S, 64 (r+1) / S) of the tile), which runs the
//                     row-pair epilogue of the GEMV kernels (bias, RoPE + KV
//                     write, SwiGLU, residual add, LM-head argmax).
// The exchange buffers are double-buffered and handed over with mbarriers in
// the peers' shared memory (arrive.release.cluster / try_wait.acquire.cluster),
// so the epilogue of tile i overlaps the main loop of tile i + 1.
//
// Across tensor-parallel ranks the row-parallel projection writes its summed
// rank-local fp32 rows to the workspace and k_tc_rows_allreduce exchanges them
// in two shots (reduce-scatter to the owner of each row pair, owner sums in
// rank order and adds the residual, all-gather of the result) as epoch-tagged
// LL words carrying bf16 pairs (P2P stores, comm.cuh).
//
// No multicast anywhere.  Every mbarrier wait is time-bounded; on a timeout the
// kernel sets its error word (jsx_device_error), the other roles of the CTA
// stop at their next wait, copies and MMAs in flight are drained (bounded) and
// TMEM is freed before the CTA exits.
#include <cuda.h>
#include <stdio.h>
#include <stdlib.h>

#include <mutex>

#include "comm.cuh"
#include "common.cuh"
#include "gemv_core.cuh"
#include "launch.cuh"
#include "tc_core.cuh"

namespace jsx {

constexpr int kTcBM = 128;  // weight rows per tile (MMA M)
constexpr int kTcBN = 32;   // tokens per tile (MMA N)
constexpr int kTcStages = 8;
constexpr int kTcThreads = 192;
constexpr int kTcMaxM = 32;
constexpr int kTcMaxCluster = 8;
constexpr int kTcMaxInvFreq = 128;  // rotary frequencies staged in shared memory by the q/k/v epilogue
constexpr uint32_t kTcABytes = kTcBM * kTcBK * 2;
constexpr uint32_t kTcBBytes = kTcBN * kTcBK * 2;
constexpr uint32_t kTcStageBytes = kTcABytes + kTcBBytes;
constexpr uint32_t kTcRingBytes = kTcStages * kTcStageBytes;
constexpr uint32_t kTcXBytes = kTcMaxM * kTcBM * 4;  // one exchange buffer: [32 tokens][128 rows] fp32
constexpr uint32_t kTcTmemCols = 64;                  // two 32-column fp32 accumulators
constexpr size_t kTcSmem = (size_t)kTcRingBytes + 2 * kTcXBytes + 1024 /* align */ + 1024 /* barriers */;

// workspace layout (bytes): kernel-done counter and argmax keys (zero between
// calls), normalised activations [32][K] bf16, rank-local rows [M][N] fp32
// (row-parallel projection across ranks)
constexpr size_t kTcOffDone = 0;
constexpr size_t kTcOffKeys = 256;
constexpr size_t kTcOffXn = 1024;

static __device__ uint32_t g_tc_error;

int read_clear_tc_error(uint32_t* out) {
  uint32_t v = 0;
  JSX_CUDA(cudaMemcpyFromSymbol(&v, g_tc_error, sizeof(v)));
  if (v) {
    const uint32_t zero = 0;
    JSX_CUDA(cudaMemcpyToSymbol(g_tc_error, &zero, sizeof(zero)));
  }
  *out = v;
  return JSX_OK;
}

struct TcArgs {
  float* part;     // [M][N] fp32 rank-local rows (store_only)
  uint32_t* done;  // CTAs finished (LM head)
  int M, N, K, kblocks, S, tiles;
  int store_only;  // write the summed rows only (k_tc_rows_allreduce finishes)
  uint64_t* trace; // null, or [grid][8] %globaltimer stamps (jsx_tc_set_trace)
};

// Per-CTA timeline: 0 entry, 1 producer issued its first ring of loads,
// 2 producer done, 3 MMA saw its first full stage, 4 MMA issued its last
// commit, 5 epilogue received its first accumulator, 6 epilogue done, 7 exit.
__device__ __forceinline__ void tc_stamp(const TcArgs& t, int k) {
  if (t.trace) t.trace[(size_t)blockIdx.x * 8 + k] = globaltimer();
}

// mbarrier wait bounded in time; a timeout raises this file's error word
template <bool kCluster = false>
__device__ __forceinline__ bool tc_wait(uint64_t* b, uint32_t parity, volatile uint32_t* abort) {
  return tc_wait_err<kCluster>(b, parity, abort, &g_tc_error);
}

constexpr uint32_t kTcIdesc = tc_idesc(kTcBM, kTcBN);

template <int EPI>
__global__ void __launch_bounds__(kTcThreads, 1) k_tc_gemm(const __grid_constant__ CUtensorMap tw,
                                                           const __grid_constant__ CUtensorMap tx, const TcArgs t,
                                                           const GemvArgs a, const CommDev c) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  float* xbuf = reinterpret_cast<float*>(smem + kTcRingBytes);  // [2][32][128]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kTcRingBytes + 2 * kTcXBytes);
  uint64_t* empty = full + kTcStages;
  uint64_t* accf = empty + kTcStages;  // [2] accumulator ready (MMA -> epilogue)
  uint64_t* acce = accf + 2;           // [2] accumulator drained (epilogue -> MMA)
  uint64_t* xfull = acce + 2;          // [2] every cluster CTA has written its exchange buffer
  uint64_t* xempty = xfull + 2;        // [2] every cluster CTA has read this CTA's exchange buffer
  uint64_t* fin = xempty + 2;          // all MMAs of the CTA complete
  unsigned long long* best = reinterpret_cast<unsigned long long*>(fin + 1);  // [32] LM-head keys
  uint32_t* misc = reinterpret_cast<uint32_t*>(best + kTcMaxM);               // tmem base, abort
  volatile uint32_t* abort_flag = misc + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = t.S;
  const uint32_t rank = cl_rank(), cid = cl_id(), ncl = cl_count();
  const int kb0 = (int)((long long)rank * t.kblocks / S);
  const int kb1 = (int)((long long)(rank + 1) * t.kblocks / S);
  if (threadIdx.x == 0) tc_stamp(t, 0);

  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s_u32(misc)),
                 "r"(kTcTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      tc_mbar_init(full + s, 1);
      tc_mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc_mbar_init(accf + b, 1);
      tc_mbar_init(acce + b, 4);
      tc_mbar_init(xfull + b, (uint32_t)S);
      tc_mbar_init(xempty + b, (uint32_t)S);
    }
    tc_mbar_init(fin, 1);
    misc[1] = 0u;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (threadIdx.x < kTcMaxM) best[threadIdx.x] = 0ull;
  tc_fence_before();
  __syncthreads();
  cl_sync_all();  // peers' barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem = misc[0];
  // Programmatic dependent launch: the next kernel may start its own prologue
  // (and weight stream) on SMs this grid frees.  Weights do not depend on the
  // previous kernel; everything it writes (activations, residual, caches) is
  // touched only after griddepcontrol.wait below.
  pdl_launch_dependents();

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      tma_prefetch_map(&tw);
      tma_prefetch_map(&tx);
      // the first ring of weight tiles goes out before the wait for the
      // previous kernel; their activation tiles follow it
      const int nkb = kb1 - kb0;
      const int pre = ((int)cid < t.tiles) ? (nkb < kTcStages ? nkb : kTcStages) : 0;
      for (int i = 0; i < pre; ++i) {
        tc_expect_tx(full + i, kTcStageBytes);
        tma_load_2d(smem + (size_t)i * kTcStageBytes, &tw, (kb0 + i) * kTcBK, (int)cid * kTcBM, full + i);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i)
        tma_load_2d(smem + (size_t)i * kTcStageBytes + kTcABytes, &tx, (kb0 + i) * kTcBK, 0, full + i);
      uint32_t it = 0;
      bool ok = true;
      for (int tile = cid; tile < t.tiles && ok; tile += ncl) {
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          if (it < (uint32_t)pre) continue;  // issued above
          const int s = it % kTcStages;
          if (it >= (uint32_t)kTcStages && !tc_wait(empty + s, ((it / kTcStages) - 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          unsigned char* st = smem + (size_t)s * kTcStageBytes;
          tc_expect_tx(full + s, kTcStageBytes);
          tma_load_2d(st, &tw, kb * kTcBK, tile * kTcBM, full + s);
          tma_load_2d(st + kTcABytes, &tx, kb * kTcBK, 0, full + s);
          if (it + 1 == (uint32_t)kTcStages) tc_stamp(t, 1);
        }
      }
      tc_stamp(t, 2);
      // every copy issued must land before the CTA exits
      const uint32_t first = it > (uint32_t)kTcStages ? it - kTcStages : 0u;
      for (uint32_t j = first; j < it; ++j) tc_wait(full + j % kTcStages, (j / kTcStages) & 1, nullptr);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t it = 0, ai = 0;
      bool ok = true;
      for (int tile = cid; tile < t.tiles && ok; tile += ncl, ++ai) {
        const uint32_t b = ai & 1;
        if (ai >= 2 && !tc_wait(acce + b, ((ai >> 1) - 1) & 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem + b * kTcBN;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % kTcStages;
          if (!tc_wait(full + s, (it / kTcStages) & 1, abort_flag)) {
            ok = false;
            break;
          }
          if (it == 0) tc_stamp(t, 3);
          tc_fence_after();
          const uint32_t sa = s_u32(smem + (size_t)s * kTcStageBytes);
          const uint32_t sb = sa + kTcABytes;
#pragma unroll
          for (int kk = 0; kk < kTcBK / 16; ++kk)
            tc_mma(d, umma_desc_sw128(sa + kk * 32), umma_desc_sw128(sb + kk * 32), kTcIdesc,
                   (kb != kb0 || kk != 0) ? 1u : 0u);
          tc_commit(empty + s);
        }
        if (ok) tc_commit(accf + b);
      }
      tc_stamp(t, 4);
      tc_commit(fin);  // arrives once every MMA issued above has completed
      tc_wait(fin, 0, nullptr);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue warps ----------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int et = threadIdx.x - 64;
    const int r = 32 * q + lane;  // tile row held after tcgen05.ld
    const int pp0 = (int)(rank * 64 / S), np = (int)((rank + 1) * 64 / S) - pp0;  // row pairs finished here
    pdl_wait();  // the epilogue reads and writes what earlier kernels use
    // q/k/v: the positions and rotary frequencies every entry reads, copied to
    // shared memory once
    const int32_t* pos_e = a.pos;
    const float* invf_e = a.inv_freq;
    if constexpr (EPI == EPI_QKV) {
      __shared__ int32_t s_pos[kTcMaxM];
      __shared__ float s_invf[kTcMaxInvFreq];
      if (!t.store_only) {
        if (et < t.M) s_pos[et] = a.pos[et];
        const int nf = a.rot >> 1;
        if (nf <= kTcMaxInvFreq)
          for (int i = et; i < nf; i += 128) s_invf[i] = a.inv_freq[i];
        epi_sync();
        pos_e = s_pos;
        if (nf <= kTcMaxInvFreq) invf_e = s_invf;
      }
    }
    uint32_t ai = 0;
    for (int tile = cid; tile < t.tiles; tile += ncl, ++ai) {
      const uint32_t b = ai & 1;
      if (!epi_all(tc_wait(accf + b, (ai >> 1) & 1, abort_flag))) break;
      if (ai == 0 && et == 0) tc_stamp(t, 5);
      tc_fence_after();
      float v[32];
      tc_ld32(tmem + ((uint32_t)(32 * q) << 16) + b * kTcBN, v);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) tc_arrive(acce + b);

      // this CTA's partial tile -> exchange buffer b (free once every peer read item ai - 2)
      if (ai >= 2 && !epi_all(tc_wait<true>(xempty + b, ((ai >> 1) - 1) & 1, abort_flag))) break;
      float* xb = xbuf + b * (kTcMaxM * kTcBM);
#pragma unroll
      for (int m = 0; m < 32; ++m)
        if (m < t.M) xb[m * kTcBM + r] = v[m];
      cl_fence();
      epi_sync();
      if (et < S) cl_arrive_remote(cl_map(s_u32(xfull + b), (uint32_t)et));
      if (!epi_all(tc_wait<true>(xfull + b, (ai >> 1) & 1, abort_flag))) break;

      // finish row pairs [pp0, pp0 + np) for every token: sum the S partials in rank order
      uint32_t src[kTcMaxCluster];
#pragma unroll
      for (int s = 0; s < kTcMaxCluster; ++s) src[s] = s < S ? cl_map(s_u32(xb), (uint32_t)s) : 0u;
      if (EPI == EPI_ROWAR && !t.store_only) {
        // single rank: h += bf16(sum); four entries at a time, every residual (and addend)
        // pair loaded before any store (no load waits behind a store it cannot be
        // proven not to alias)
        for (int e0 = et; e0 < np * t.M; e0 += 4 * 128) {
          float v0[4], v1[4];
          uint32_t hv[4], ad[4];
          size_t idx[4];
          bool ok[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int e = e0 + 128 * u;
            ok[u] = false;
            v0[u] = v1[u] = 0.f;
            idx[u] = 0;
            if (e < np * t.M) {
              const int m = e / np, p = pp0 + (e - m * np);
              const uint32_t off = (uint32_t)(m * kTcBM + 2 * p) * 4u;
#pragma unroll
              for (int s = 0; s < kTcMaxCluster; ++s) {
                if (s < S) {
                  const float2 f = cl_ld2(src[s] + off);
                  v0[u] += f.x;
                  v1[u] += f.y;
                }
              }
              const int row0 = tile * kTcBM + 2 * p;
              ok[u] = row0 < t.N;
              idx[u] = (size_t)m * t.N + row0;
            }
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            hv[u] = ok[u] ? *reinterpret_cast<const uint32_t*>(a.h + idx[u]) : 0u;
            ad[u] = (ok[u] && a.addend) ? *reinterpret_cast<const uint32_t*>(a.addend + idx[u]) : 0u;
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (!ok[u]) continue;
            float w0 = v0[u], w1 = v1[u];
            if (a.addend) {
              w0 += __uint_as_float(ad[u] << 16);
              w1 += __uint_as_float(ad[u] & 0xffff0000u);
            }
            *reinterpret_cast<uint32_t*>(a.h + idx[u]) =
                pack2(__uint_as_float(hv[u] << 16) + rbf(w0), __uint_as_float(hv[u] & 0xffff0000u) + rbf(w1));
          }
        }
      } else {
        // four entries at a time: their partial sums (and q/k/v bias pairs) are
        // all loaded before any entry's epilogue, so the loads of one batch
        // share a round trip instead of one per entry
        for (int e0 = et; e0 < np * t.M; e0 += 4 * 128) {
          float v0[4], v1[4], b0[4], b1[4];
          int mm[4], rr[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int e = e0 + 128 * u;
            v0[u] = v1[u] = b0[u] = b1[u] = 0.f;
            mm[u] = 0;
            rr[u] = -1;
            if (e < np * t.M) {
              const int m = e / np, p = pp0 + (e - m * np);
              const uint32_t off = (uint32_t)(m * kTcBM + 2 * p) * 4u;
#pragma unroll
              for (int s = 0; s < kTcMaxCluster; ++s) {
                if (s < S) {
                  const float2 f = cl_ld2(src[s] + off);
                  v0[u] += f.x;
                  v1[u] += f.y;
                }
              }
              const int row0 = tile * kTcBM + 2 * p;
              if (row0 < t.N) {
                rr[u] = row0;
                mm[u] = m;
                if (EPI == EPI_QKV && !t.store_only) qkv_bias_pair(a, row0 >> 1, b0[u], b1[u]);
              }
            }
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (rr[u] < 0) continue;
            const int m = mm[u], row0 = rr[u];
            if (t.store_only) {
              t.part[(size_t)m * t.N + row0] = v0[u];
              t.part[(size_t)m * t.N + row0 + 1] = v1[u];
            } else if constexpr (EPI == EPI_QKV) {
              qkv_store_b(a, row0 >> 1, m, v0[u], v1[u], b0[u], b1[u], pos_e, invf_e);
            } else {
              const unsigned long long key = epi_pair<EPI>(a, c, false, 0u, row0 >> 1, m, v0[u], v1[u]);
              if (EPI == EPI_LMHEAD && key) atomicMax(best + m, key);
            }
          }
        }
      }
      epi_sync();  // every read of the peers' buffers is complete
      if (et < S) cl_arrive_remote(cl_map(s_u32(xempty + b), (uint32_t)et));
    }
    if (et == 0) tc_stamp(t, 6);
    __syncwarp();
  }

  // ---------------- teardown ----------------
  pdl_wait();
  tc_fence_before();
  __syncthreads();
  cl_sync_all();  // no CTA leaves while a peer may still read its exchange buffers
  if (threadIdx.x == 0) tc_stamp(t, 7);
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcTmemCols)
                 : "memory");
  }
  if constexpr (EPI == EPI_LMHEAD) {
    if (threadIdx.x < t.M && best[threadIdx.x]) atomicMax(a.keys + threadIdx.x, best[threadIdx.x]);
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) misc[2] = (atomicAdd(t.done, 1u) == gridDim.x - 1) ? 1u : 0u;
    __syncthreads();
    if (!misc[2]) return;
    __threadfence();
    unsigned long long* fk = best;  // reuse: final keys [32]
    if (threadIdx.x < t.M) fk[threadIdx.x] = atomicAdd(a.keys + threadIdx.x, 0ull);
    __syncthreads();
    if (c.world > 1) {
      const uint32_t ep = read_epoch(c);
      const int pr = ep & 1;
      if (threadIdx.x < t.M)
        for (int d = 0; d < c.world; ++d) key_ptr(c, d, pr, c.rank)[threadIdx.x] = fk[threadIdx.x];
      __threadfence_system();
      __syncthreads();
      if (threadIdx.x < c.world) st_release_sys(flag_ptr(c, threadIdx.x, kMaxCtas, c.rank), ep);
      if (threadIdx.x < c.world) wait_flag(c, kMaxCtas, threadIdx.x, ep);
      __syncthreads();
      if (threadIdx.x < t.M) {
        unsigned long long bk = 0ull;
        for (int s = 0; s < c.world; ++s) {
          const unsigned long long k = __ldcg(key_ptr(c, c.rank, pr, s) + threadIdx.x);
          bk = k > bk ? k : bk;
        }
        fk[threadIdx.x] = bk;
      }
      __syncthreads();
      if (threadIdx.x == 0) c.state[kCalls] = ep;
    }
    if (threadIdx.x < t.M) {
      a.ids[threadIdx.x] = (int32_t)argmax_key_index(fk[threadIdx.x]);
      a.keys[threadIdx.x] = 0ull;
    }
    if (threadIdx.x == 0) *t.done = 0u;
  }
}

// ---- row-parallel projection across ranks: NVLink all-reduce + residual --------
// CTA b owns row pairs [p0, p1); pushes this rank's fp32 rows to every rank's
// LL slots, then reads its rows from every rank's slots once they carry the
// call's epoch, sums them in rank order and adds the residual (comm.cuh).
// Two-shot exchange of the rank-local fp32 rows `part` [M][N] that k_tc_gemm
// (store_only) left in the workspace, as epoch-tagged LL words whose payload is
// a bf16 pair (each rank's partial rounded to bf16, the reference's per-rank
// result; the wide path rounds the same way):
//   reduce-scatter: row pair g belongs to rank g / ppr; every rank stores its
//     packed partial of pair g into the owner's slot [source rank][m][g - owner ppr];
//   the owner sums the ranks' bf16 partials in fp32 in rank order, adds the
//     residual, rounds once (h is then identical on every rank), stores h and
//     pushes the packed result into every peer's gather slot [m][g];
//   gather: the pairs other ranks own are read from the gather slots into h.
// Each rank sends 2 x (world - 1) / world x M x N / 2 words, against world x M x N
// words for a one-shot push of fp32 partials.  Waits: an owner waits only for
// pushes that never wait; a gather waits only for owners.  Every CTA has
// started (PDL trigger at entry) before a dependent kernel may occupy an SM.
// Slots: the comm's LL words of the call's parity, gather slots after the
// world x max_tokens x hidden / 2 reduce-scatter slots.
__device__ __forceinline__ void ll_put_raw(unsigned long long* slot, uint32_t payload, uint32_t epoch) {
  const unsigned long long w = ((unsigned long long)epoch << 32) | payload;
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(slot), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ll_load_raw(const unsigned long long* slot) {
  unsigned long long w;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(slot) : "memory");
  return w;
}
// bounded poll of one slot for `epoch`; on timeout the comm's error word is set and 0 returned
__device__ __noinline__ uint32_t ll_wait_raw(uint32_t* state, unsigned long long timeout_ns,
                                             const unsigned long long* slot, uint32_t epoch) {
  if (*reinterpret_cast<volatile uint32_t*>(state + kError)) return 0u;
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    const unsigned long long w = ll_load_raw(slot);
    if ((uint32_t)(w >> 32) == epoch) return (uint32_t)w;
    if ((it & 15u) == 0) {
      if (globaltimer() - t0 > timeout_ns || it > (1u << 28)) {
        atomicOr(state + kError, 1u);
        return 0u;
      }
      __nanosleep(20);
    }
  }
}

// Rank-ordered sums of one bf16 pair's LL slots (source src at p0 + src *
// sstride) once all carry `epoch`: every slot still without it is reloaded,
// all in flight together (one round trip per pass).  Bounded: on timeout (or
// when an earlier wait of this rank gave up) the error word is set and the
// missing slots count as 0.
__device__ __noinline__ float2 ll_sum_pairs_poll(uint32_t* state, unsigned long long timeout_ns,
                                                 const unsigned long long* p0, size_t sstride, int W,
                                                 uint32_t epoch) {
  unsigned long long w[kMaxRanks];
#pragma unroll
  for (int src = 0; src < kMaxRanks; ++src) w[src] = 0ull;
  const uint64_t t0 = globaltimer();
  bool all = false;
#pragma unroll 1
  for (uint32_t it = 1; !all; ++it) {
#pragma unroll
    for (int src = 0; src < kMaxRanks; ++src)
      if (src < W && (uint32_t)(w[src] >> 32) != epoch) w[src] = ll_load_raw(p0 + src * sstride);
    all = true;
#pragma unroll
    for (int src = 0; src < kMaxRanks; ++src)
      if (src < W) all = all && (uint32_t)(w[src] >> 32) == epoch;
    if (!all && (it & 15u) == 0) {
      if (*reinterpret_cast<volatile uint32_t*>(state + kError)) break;
      if (globaltimer() - t0 > timeout_ns || it > (1u << 28)) {
        atomicOr(state + kError, 1u);
        break;
      }
      __nanosleep(20);
    }
  }
  float s0 = 0.f, s1 = 0.f;
#pragma unroll
  for (int src = 0; src < kMaxRanks; ++src) {
    if (src < W) {
      const uint32_t pv = (uint32_t)(w[src] >> 32) == epoch ? (uint32_t)w[src] : 0u;
      s0 += __uint_as_float(pv << 16);
      s1 += __uint_as_float(pv & 0xffff0000u);
    }
  }
  return make_float2(s0, s1);
}

__global__ void __launch_bounds__(256) k_tc_rows_allreduce(GemvArgs a, const float* __restrict__ part, CommDev c) {
  pdl_wait();
  pdl_launch_dependents();
  const int M = a.M, NB = a.N >> 1, W = c.world;
  const int ppr = (NB + W - 1) / W;  // row pairs per owner
  const uint32_t epoch = read_epoch(c);
  const int par = epoch & 1;
  const size_t rs_words = (size_t)W * c.max_tokens * (c.hidden >> 1);
  const int nthreads = gridDim.x * blockDim.x, tid = blockIdx.x * blockDim.x + threadIdx.x;
  // reduce-scatter pushes
  for (int e = tid; e < M * NB; e += nthreads) {
    const int m = e / NB, g = e - m * NB;
    const float2 v = __ldcg(reinterpret_cast<const float2*>(part + (size_t)m * a.N + 2 * g));
    const int d = g / ppr;
    unsigned long long* slot = data_ptr(c, d, par, 0, 0) + ((size_t)c.rank * c.max_tokens + m) * ppr + (g - d * ppr);
    ll_put_raw(slot, pack2(v.x, v.y), epoch);
  }
  // owner: sum the ranks' partials of the pairs this rank owns, residual, push the result
  const int g0 = c.rank * ppr, gn = max(0, min(NB, g0 + ppr) - g0);  // pairs [g0, g0 + gn) are this rank's
  const unsigned long long* mine = data_ptr(c, c.rank, par, 0, 0);
  for (int e = tid; e < M * gn; e += nthreads) {
    const int m = e / gn, pl = e - m * gn, g = g0 + pl;
    uint32_t* hp = reinterpret_cast<uint32_t*>(a.h + (size_t)m * a.N + 2 * g);
    const uint32_t hv = *hp;
    unsigned long long w[kMaxRanks];
#pragma unroll
    for (int src = 0; src < kMaxRanks; ++src)
      if (src < W) w[src] = ll_load_raw(mine + ((size_t)src * c.max_tokens + m) * ppr + pl);
    float s0 = 0.f, s1 = 0.f;
    bool all = true;
#pragma unroll
    for (int src = 0; src < kMaxRanks; ++src) {
      if (src < W) {
        all = all && (uint32_t)(w[src] >> 32) == epoch;
        s0 += __uint_as_float((uint32_t)w[src] << 16);
        s1 += __uint_as_float((uint32_t)w[src] & 0xffff0000u);
      }
    }
    if (!all) {
      const float2 sp = ll_sum_pairs_poll(c.state, c.timeout_ns, mine + (size_t)m * ppr + pl,
                                          (size_t)c.max_tokens * ppr, W, epoch);
      s0 = sp.x;
      s1 = sp.y;
    }
    const uint32_t hn = pack2(__uint_as_float(hv << 16) + rbf(s0), __uint_as_float(hv & 0xffff0000u) + rbf(s1));
    *hp = hn;
    for (int d = 0; d < W; ++d)
      if (d != c.rank) ll_put_raw(data_ptr(c, d, par, 0, 0) + rs_words + (size_t)m * (c.hidden >> 1) + g, hn, epoch);
  }
  // gather the pairs the other ranks own
  const int others = NB - gn;
  for (int e = tid; e < M * others; e += nthreads) {
    const int m = e / others, k = e - m * others;
    const int g = k < g0 ? k : k + gn;
    const unsigned long long* slot = mine + rs_words + (size_t)m * (c.hidden >> 1) + g;
    const unsigned long long w = ll_load_raw(slot);
    const uint32_t hn = (uint32_t)(w >> 32) == epoch ? (uint32_t)w : ll_wait_raw(c.state, c.timeout_ns, slot, epoch);
    *reinterpret_cast<uint32_t*>(a.h + (size_t)m * a.N + 2 * g) = hn;
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

// ---- host ------------------------------------------------------------------------

// Cluster launch of k_tc_gemm; programmatic dependent launch when the
// library's launch flags ask for it (attr holds 2 entries).
static cudaLaunchConfig_t tc_config(int grid, int S, cudaStream_t s, cudaLaunchAttribute* attr, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = kTcSmem;
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cfg;
}

// Clusters of S CTAs that fit on the device at once (one CTA per SM), per
// device; without a device, 148 / S (a B200).
static int max_clusters(int S) {
  static int cache[64][kTcMaxCluster + 1] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return 148 / S;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev][S] == 0) {
    int n = 0;
    auto kern = k_tc_gemm<EPI_LINEAR>;
    cudaLaunchAttribute attr[2];
    cudaLaunchConfig_t cfg = tc_config(S, S, nullptr, attr, false);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem) != cudaSuccess ||
        cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n < 1) {
      cudaGetLastError();
      n = sm_count() / S;
    }
    cache[dev][S] = n > 0 ? n : 1;
  }
  return cache[dev][S];
}

struct TcPlan {
  int tiles, kblocks, S, clusters;
  size_t part_off, bytes;
};

// Cluster size S = 1..min(8, K blocks): the smallest modelled time
//   waves x (K blocks per CTA x 20 KB + 16 KB of per-tile cost),
// waves = ceil(tiles / clusters resident at once); ties keep the smaller S.
static TcPlan tc_plan(int M, int K, int N) {
  TcPlan p;
  p.tiles = (N + kTcBM - 1) / kTcBM;
  p.kblocks = (K + kTcBK - 1) / kTcBK;
  const int smax = p.kblocks < kTcMaxCluster ? p.kblocks : kTcMaxCluster;
  long long best_cost = -1;
  p.S = 1;
  p.clusters = 1;
  for (int s = 1; s <= smax; ++s) {
    const int cl = max_clusters(s);
    const long long waves = (p.tiles + cl - 1) / cl;
    const long long per = (p.kblocks + s - 1) / s;
    const long long cost = waves * (per * 20480 + 16384);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      p.S = s;
      p.clusters = cl < p.tiles ? cl : p.tiles;
    }
  }
  p.part_off = kTcOffXn + (((size_t)kTcMaxM * K * 2 + 1023) & ~(size_t)1023);
  p.bytes = p.part_off + (size_t)M * N * sizeof(float);
  return p;
}

CommDev comm_view(jsx_comm* comm);

static uint64_t* g_trace_buf = nullptr;  // jsx_tc_set_trace
uint64_t* tc_trace_buffer() { return g_trace_buf; }  // also stamped by the wide GEMM (tc_wide.cu)

template <int EPI>
static int tc_run(jsx_comm* comm, GemvArgs ga, void* workspace, size_t workspace_bytes, cudaStream_t s) {
  JSX_REQUIRE(ga.M >= 1 && ga.M <= kTcMaxM, "M=%d outside 1..%d", ga.M, kTcMaxM);
  JSX_REQUIRE(ga.K >= 8 && ga.K % 8 == 0, "K=%d must be a positive multiple of 8", ga.K);
  JSX_REQUIRE(ga.N >= 2 && ga.N % 2 == 0, "N=%d must be even", ga.N);
  JSX_REQUIRE(aligned16(ga.x) && aligned16(ga.w), "activation and weight must be 16-byte aligned");
  const TcPlan p = tc_plan(ga.M, ga.K, ga.N);
  JSX_REQUIRE(workspace && aligned16(workspace) && workspace_bytes >= p.bytes,
              "workspace of %zu bytes (16-byte aligned) required", p.bytes);
  unsigned char* ws = (unsigned char*)workspace;
  CommDev c = {};
  c.world = 1;
  if (comm) {
    c = comm_view(comm);
    JSX_REQUIRE(ga.M <= c.max_tokens && (EPI != EPI_ROWAR || ga.N <= c.hidden),
                "M=%d N=%d exceed the comm buffer", ga.M, ga.N);
  }
  if (EPI == EPI_LMHEAD) {
    ga.done = (uint32_t*)(ws + kTcOffDone);
    ga.keys = (unsigned long long*)(ws + kTcOffKeys);
  }
  // activations: RMS-normalised copy when a gain is given (layers/normalization.py:31-37)
  const void* x = ga.x;
  if (ga.gamma) {
    const int st = jsx_rmsnorm(ga.x, ga.gamma, ws + kTcOffXn, ga.M, ga.K, ga.eps, s);
    if (st) return st;
    x = ws + kTcOffXn;
  }
  CUtensorMap tw, tx;
  int st = make_map(&tw, ga.w, ga.N, ga.K, kTcBM);
  if (st) return st;
  st = make_map(&tx, x, ga.M, ga.K, kTcBN);
  if (st) return st;
  const bool across_ranks = EPI == EPI_ROWAR && c.world > 1;
  TcArgs ta;
  ta.part = (float*)(ws + p.part_off);
  ta.done = (uint32_t*)(ws + kTcOffDone);
  ta.M = ga.M; ta.N = ga.N; ta.K = ga.K; ta.kblocks = p.kblocks; ta.S = p.S; ta.tiles = p.tiles;
  ta.store_only = across_ranks ? 1 : 0;
  ta.trace = g_trace_buf;
  auto kern = k_tc_gemm<EPI>;
  JSX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem));
  cudaLaunchAttribute attr[2];
  const cudaLaunchConfig_t cfg = tc_config(p.clusters * p.S, p.S, s, attr, (launch_flags() & JSX_LAUNCH_PDL) != 0);
  JSX_CUDA(cudaLaunchKernelEx(&cfg, kern, tw, tx, ta, ga, c));
  if (across_ranks) {
    int rgrid = 2 * sm_count();
    if (rgrid > kMaxCtas) rgrid = kMaxCtas;
    if (rgrid > ga.N / 2) rgrid = ga.N / 2;
    JSX_CUDA(launch_kernel(k_tc_rows_allreduce, dim3(rgrid), dim3(256), 0, s, ga, ta.part, c));
  }
  return JSX_OK;
}

}  // namespace jsx

using namespace jsx;

extern "C" int jsx_tc_set_trace(uint64_t* buf) {
  g_trace_buf = buf;
  return JSX_OK;
}

extern "C" int jsx_tc_workspace_size(int M, int K, int N, size_t* bytes) {
  JSX_REQUIRE(bytes && M >= 1 && M <= kTcMaxM && K >= 8 && N >= 2, "bad arguments");
  *bytes = tc_plan(M, K, N).bytes;
  return JSX_OK;
}

extern "C" int jsx_tc_linear(const void* x, const void* gamma, float eps, const void* w_nk, const void* bias, void* y,
                             int M, int K, int N, void* workspace, size_t workspace_bytes, void* stream) {
  JSX_REQUIRE(x && w_nk && y, "null pointer argument");
  GemvArgs a = {};
  a.x = (const bf16*)x; a.gamma = (const bf16*)gamma; a.eps = eps; a.w = (const bf16*)w_nk;
  a.M = M; a.K = K; a.N = N; a.bias = (const bf16*)bias; a.y = (bf16*)y;
  return tc_run<EPI_LINEAR>(nullptr, a, workspace, workspace_bytes, (cudaStream_t)stream);
}

extern "C" int jsx_tc_qkv_rope_cache(const void* h, const void* ln_gamma, float eps, const void* w_qkv,
                                     const void* b_qkv, const float* inv_freq, const int32_t* positions,
                                     void* q_out, void* k_cache, void* v_cache, int M, int tokens_per_seq, int K,
                                     int nq, int nkv, int head_dim, int rotary_dim, int max_seq, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  JSX_REQUIRE(h && w_qkv && q_out && k_cache && v_cache && positions && inv_freq, "null pointer argument");
  JSX_REQUIRE(head_dim >= 2 && head_dim % 2 == 0 && rotary_dim >= 0 && rotary_dim <= head_dim &&
                  rotary_dim % 2 == 0 && (head_dim - rotary_dim) % 2 == 0,
              "head_dim=%d rotary_dim=%d", head_dim, rotary_dim);
  JSX_REQUIRE(tokens_per_seq >= 1 && M % tokens_per_seq == 0 && max_seq >= 1, "bad tokens_per_seq/max_seq");
  GemvArgs a = {};
  a.x = (const bf16*)h; a.gamma = (const bf16*)ln_gamma; a.eps = eps; a.w = (const bf16*)w_qkv;
  a.M = M; a.K = K; a.N = (nq + 2 * nkv) * head_dim; a.bias = (const bf16*)b_qkv; a.y = (bf16*)q_out;
  a.inv_freq = inv_freq; a.pos = positions; a.kc = (bf16*)k_cache; a.vc = (bf16*)v_cache;
  a.nq = nq; a.nkv = nkv; a.hd = head_dim; a.rot = rotary_dim; a.max_seq = max_seq; a.tps = tokens_per_seq;
  return tc_run<EPI_QKV>(nullptr, a, workspace, workspace_bytes, (cudaStream_t)stream);
}

extern "C" int jsx_tc_gate_up_swiglu(const void* h, const void* ln_gamma, float eps, const void* w_gu, void* act,
                                     int M, int K, int I, void* workspace, size_t workspace_bytes, void* stream) {
  JSX_REQUIRE(h && w_gu && act, "null pointer argument");
  GemvArgs a = {};
  a.x = (const bf16*)h; a.gamma = (const bf16*)ln_gamma; a.eps = eps; a.w = (const bf16*)w_gu;
  a.M = M; a.K = K; a.N = 2 * I; a.y = (bf16*)act;
  return tc_run<EPI_SWIGLU>(nullptr, a, workspace, workspace_bytes, (cudaStream_t)stream);
}

extern "C" int jsx_tc_row_linear_allreduce(jsx_comm* comm, const void* x, const void* w_nk, void* h, int M,
                                           int K_local, int N, void* workspace, size_t workspace_bytes,
                                           void* stream) {
  JSX_REQUIRE(x && w_nk && h, "null pointer argument");
  GemvArgs a = {};
  a.x = (const bf16*)x; a.w = (const bf16*)w_nk; a.M = M; a.K = K_local; a.N = N; a.h = (bf16*)h;
  return tc_run<EPI_ROWAR>(comm, a, workspace, workspace_bytes, (cudaStream_t)stream);
}

extern "C" int jsx_tc_lmhead_argmax(jsx_comm* comm, const void* h, const void* norm_gamma, float eps,
                                    const void* w_vocab, int vocab_local, int vocab_offset, int M, int hidden,
                                    void* logits_out, int32_t* ids_out, void* workspace, size_t workspace_bytes,
                                    void* stream) {
  JSX_REQUIRE(h && w_vocab && ids_out && vocab_offset >= 0, "bad arguments");
  GemvArgs a = {};
  a.x = (const bf16*)h; a.gamma = (const bf16*)norm_gamma; a.eps = eps; a.w = (const bf16*)w_vocab;
  a.M = M; a.K = hidden; a.N = vocab_local; a.y = (bf16*)logits_out; a.vocab_offset = vocab_offset;
  a.ids = ids_out;
  return tc_run<EPI_LMHEAD>(comm, a, workspace, workspace_bytes, (cudaStream_t)stream);
}
