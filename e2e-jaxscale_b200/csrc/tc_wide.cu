// Wide tensor-core GEMM for many tokens: prefill projections and row-parallel
// products of 64 and more tokens (tcgen05 + TMA).  y[tokens][rows] = x W^T with
// the decode projections' pair epilogues (bias, RoPE + KV write, SwiGLU,
// residual add), for the reference's LinearBase.__call__ (layers/linear.py:57-82)
// over [B, S] token blocks (models/glm4.py:97-132 at prefill).
//
// Tile: D[128 weight rows, 256 tokens]; the weight box [128][64] is the MMA's A
// operand (M = 128), the token box [256][64] its B operand (N = 256), both
// K-major bf16 with the 128-byte swizzle, staged by TMA in a 4-stage ring of
// 48 KB stages; fp32 accumulation in TMEM with two accumulators of 256 columns
// (the whole TMEM of the SM: one CTA per SM, which the shared memory enforces).
// A 128 x 256 x 64 stage is 4 MMAs of K = 16 and 4.2 MFLOP per 48 KB staged.
//
// Persistent CTAs walk the tiles in groups of kWGroup token tiles; inside a
// group the tiles are ordered weight-tile-major, so CTAs running at the same
// time share weight tiles and the group's token tiles stay in L2 while the
// weight matrix passes once per group.
//
// Roles: warp 0 / lane 0 TMA producer, warp 1 / lane 0 MMA issuer, warps 2..5
// epilogue: tcgen05.ld 32x32b.x32 (lane = weight row, 32 tokens per chunk),
// row pairs (2g, 2g+1) formed with one shuffle per token (the even lane takes
// tokens 0..15 of the chunk, the odd lane 16..31), then the pair epilogue of
// the decode kernels.  The accumulator is handed back after the tile's last
// chunk is read, so the epilogue of tile i overlaps the main loop of i + 1.
//
// No multicast.  Every mbarrier wait is time-bounded; on a timeout the kernel
// sets its error word (jsx_device_error), the other roles stop at their next
// wait, copies and MMAs in flight are drained (bounded) and TMEM is freed.
#include "comm.cuh"
#include "common.cuh"
#include "gemv_core.cuh"
#include "launch.cuh"
#include "tc_core.cuh"

namespace jsx {

constexpr int kWBM = 128;     // weight rows per tile (MMA M)
constexpr int kWBN = 256;     // tokens per tile (MMA N)
constexpr int kWStages = 4;
constexpr int kWThreads = 192;
constexpr int kWGroup = 8;    // token tiles per group of the tile order
constexpr uint32_t kWABytes = kWBM * kTcBK * 2;
constexpr uint32_t kWBBytes = kWBN * kTcBK * 2;
constexpr uint32_t kWStageBytes = kWABytes + kWBBytes;
constexpr uint32_t kWRingBytes = kWStages * kWStageBytes;
constexpr uint32_t kWTmemCols = 2 * kWBN;
constexpr uint32_t kWStageOff = kWRingBytes + 1024;  // after the ring and the barriers
constexpr size_t kWSmem = (size_t)kWStageOff + 4 * 32 * 32 * 2 /* exchange staging */ + 1024 /* align */;
constexpr uint32_t kWIdesc = tc_idesc(kWBM, kWBN);
constexpr size_t kWOffXn = 1024;  // workspace: header, then the RMS-normalised activations [M][K] bf16

static_assert(kWBN % 32 == 0 && kWBN <= 256, "token tile: MMA N and TMA box limit");
static_assert(kWTmemCols <= 512, "two accumulators in the SM's TMEM");
static_assert(kWBM == kXTileRows && kWBN == kXTileTokens && kWBM == 32 * kXQuarters,
              "the tile exchange's slots hold one output tile, one quarter per epilogue warp");

static __device__ uint32_t g_wide_error;

int read_clear_wide_error(uint32_t* out) {
  uint32_t v = 0;
  JSX_CUDA(cudaMemcpyFromSymbol(&v, g_wide_error, sizeof(v)));
  if (v) {
    const uint32_t zero = 0;
    JSX_CUDA(cudaMemcpyToSymbol(g_wide_error, &zero, sizeof(zero)));
  }
  *out = v;
  return JSX_OK;
}

template <bool kCluster = false>
__device__ __forceinline__ bool w_wait(uint64_t* b, uint32_t parity, volatile uint32_t* abort) {
  return tc_wait_err<kCluster>(b, parity, abort, &g_wide_error);
}

struct WideArgs {
  int M, N, K, kblocks;
  int ntt, nft, tiles;  // token tiles, weight tiles, ntt * nft
  uint64_t* trace;      // null, or [grid][8] %globaltimer stamps (jsx_tc_set_trace): 0 entry,
                        // 1 first accumulator at the epilogue, 2 epilogue done with the tiles
                        // other ranks own, 3 with every tile, 4 finished tiles gathered,
                        // 5 last MMA commit, 6 last TMA load issued, 7 exit
};

__device__ __forceinline__ void wide_stamp(const WideArgs& t, int k) {
  if (t.trace) t.trace[(size_t)blockIdx.x * 8 + k] = globaltimer();
}

// tile -> (weight tile ft, token tile tt): groups of kWGroup token tiles,
// weight-tile-major inside a group
__device__ __forceinline__ void wide_tile(const WideArgs& t, int tile, int& ft, int& tt) {
  const int per_group = kWGroup * t.nft;
  const int grp = tile / per_group;
  const int rem = tile - grp * per_group;
  const int left = t.ntt - grp * kWGroup;
  const int gsz = left < kWGroup ? left : kWGroup;
  ft = rem / gsz;
  tt = grp * kWGroup + (rem - ft * gsz);
}

// Pair epilogue (rows 2g, 2g+1 of token m) with packed 4-byte stores where the
// two rows are adjacent in the output; the arithmetic is the decode kernels'.
template <int EPI>
__device__ __forceinline__ void wide_pair(const GemvArgs& a, int g, int m, float v0, float v1, float b0, float b1) {
  const int r0 = 2 * g;
  if constexpr (EPI == EPI_LINEAR) {
    float y0 = rbf(v0), y1 = rbf(v1);
    if (a.bias) {
      y0 = rbf(y0 + b0);
      y1 = rbf(y1 + b1);
    }
    *reinterpret_cast<uint32_t*>(a.y + (size_t)m * a.N + r0) = pack2(y0, y1);
  } else if constexpr (EPI == EPI_QKV) {
    qkv_store(a, g, m, v0, v1);
  } else if constexpr (EPI == EPI_SWIGLU) {
    swiglu_store(a, g, m, v0, v1);
  } else if constexpr (EPI == EPI_ROWAR) {
    if (a.addend) {
      const uint32_t ad = *reinterpret_cast<const uint32_t*>(a.addend + (size_t)m * a.N + r0);
      v0 += __uint_as_float(ad << 16);
      v1 += __uint_as_float(ad & 0xffff0000u);
    }
    uint32_t* hp = reinterpret_cast<uint32_t*>(a.h + (size_t)m * a.N + r0);
    const uint32_t hv = *hp;
    *hp = pack2(__uint_as_float(hv << 16) + rbf(v0), __uint_as_float(hv & 0xffff0000u) + rbf(v1));
  }
}

__device__ __forceinline__ void pack8(const float (&f)[8], uint4& u) {
  u.x = pack2(f[0], f[1]);
  u.y = pack2(f[2], f[3]);
  u.z = pack2(f[4], f[5]);
  u.w = pack2(f[6], f[7]);
}

// One epilogue warp's quarter (32 rows x 256 tokens) of a tile in the
// single-rank row-parallel product (h += bf16(partial)): per 32-token chunk the
// bf16-rounded partials are transposed through shared memory into
// [token][32 rows], so the residual is read and written with 16-byte accesses
// (4 per lane and chunk instead of 16 four-byte ones: the load/store issue rate,
// not the tensor cores, bounded this epilogue at small K), the next chunk's
// residual loaded ahead of this chunk's stores.  Same arithmetic as wide_pair:
// h + bf16(v) in fp32, rounded once.
__device__ __forceinline__ void wide_rowar_tile(const WideArgs& t, const GemvArgs& a, int ft, int tt, int q, int lane,
                                                uint32_t tacc, uint64_t* acc_empty, bf16* stg) {
  const int r0 = ft * kWBM + 32 * q;
  uint4 hv[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int e = lane + 32 * k;
    const int m = tt * kWBN + (e >> 2), row = r0 + 8 * (e & 3);
    hv[k] = (m < t.M && row < t.N) ? *reinterpret_cast<const uint4*>(a.h + (size_t)m * t.N + row)
                                   : make_uint4(0, 0, 0, 0);
  }
#pragma unroll 1
  for (int ch = 0; ch < kWBN / 32; ++ch) {
    float v[32];
    tc_ld32(tacc + 32 * ch, v);
    if (ch == kWBN / 32 - 1) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) tc_arrive(acc_empty);
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) stg[j * 32 + lane] = __float2bfloat16_rn(v[j]);
    __syncwarp();
    uint4 hn[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int e = lane + 32 * k;
      const int m = tt * kWBN + 32 * (ch + 1) + (e >> 2), row = r0 + 8 * (e & 3);
      hn[k] = (ch + 1 < kWBN / 32 && m < t.M && row < t.N)
                  ? *reinterpret_cast<const uint4*>(a.h + (size_t)m * t.N + row)
                  : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int e = lane + 32 * k;
      const int m = tt * kWBN + 32 * ch + (e >> 2), row = r0 + 8 * (e & 3);
      if (m >= t.M || row >= t.N) continue;
      float hf[8], pf[8];
      unpack8(hv[k], hf);
      unpack8(*reinterpret_cast<const uint4*>(stg + (e >> 2) * 32 + 8 * (e & 3)), pf);
#pragma unroll
      for (int i = 0; i < 8; ++i) hf[i] += pf[i];
      uint4 o;
      pack8(hf, o);
      *reinterpret_cast<uint4*>(a.h + (size_t)m * t.N + row) = o;
    }
    __syncwarp();  // the staging buffer is refilled by the next chunk
#pragma unroll
    for (int k = 0; k < 4; ++k) hv[k] = hn[k];
  }
}

// One epilogue warp's quarter (32 rows x 256 tokens) of a tile in the
// row-parallel product across ranks.  Per 32-token chunk the accumulator is
// rounded to bf16 (this rank's partial, the reference's per-rank result) and
// transposed through shared memory into [token][32 rows], so that every
// transfer is a 16-byte store and a quarter is 16 KB contiguous:
//   not the owner: push the partial into the owner's slot, then flag it;
//   owner: wait for the peers' partials, sum the ranks' bf16 partials in fp32
//   in rank order, round, add the residual (identical h on every rank), store
//   h here and the finished quarter into every peer's result array, flag them.
__device__ __forceinline__ void wide_exchange_tile(const CommDev& c, const WideArgs& t, const GemvArgs& a, int tile,
                                                   int ft, int tt, int q, int lane, uint32_t epoch, uint32_t tacc,
                                                   uint64_t* acc_empty, bf16* stg) {
  const int owner = tile % c.world, jo = tile / c.world;
  const bool mine = owner == c.rank;
  if (mine)
    for (int src = 0; src < c.world; ++src)
      if (src != c.rank) wait_epoch_sys(c, pflag_ptr(c, c.rank, jo, src, q), epoch);
  bf16* push = mine ? nullptr : slot_ptr(c, owner, jo, c.rank, q);
#pragma unroll 1
  for (int ch = 0; ch < kWBN / 32; ++ch) {
    float v[32];
    tc_ld32(tacc + 32 * ch, v);
    if (ch == kWBN / 32 - 1) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) tc_arrive(acc_empty);
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) stg[j * 32 + lane] = __float2bfloat16_rn(v[j]);
    __syncwarp();
    // this lane's 4 vectors of the chunk: vector e = lane + 32 k is token e / 4,
    // rows 8 (e % 4) .. + 7 of the quarter
    uint4 part[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int e = lane + 32 * k;
      part[k] = *reinterpret_cast<const uint4*>(stg + (e >> 2) * 32 + 8 * (e & 3));
    }
    const int mlc = 32 * ch;  // first token of the chunk inside the tile
    if (!mine) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int e = lane + 32 * k;
        *reinterpret_cast<uint4*>(push + (mlc + (e >> 2)) * 32 + 8 * (e & 3)) = part[k];
      }
    } else {
      // every load of the chunk is issued before any store (one round trip per source)
      uint4 hv[4];
      bool live[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int e = lane + 32 * k;
        const int m = tt * kWBN + mlc + (e >> 2), row = ft * kWBM + 32 * q + 8 * (e & 3);
        live[k] = m < t.M && row < t.N;
        hv[k] = live[k] ? *reinterpret_cast<const uint4*>(a.h + (size_t)m * t.N + row) : make_uint4(0, 0, 0, 0);
      }
      float sum[4][8];
#pragma unroll
      for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int i = 0; i < 8; ++i) sum[k][i] = 0.f;
      // four sources' slots loaded at a time, then summed in rank order
      for (int s0 = 0; s0 < c.world; s0 += 4) {
        uint4 u[4][4];
#pragma unroll
        for (int sj = 0; sj < 4; ++sj) {
          const int src = s0 + sj;
          if (src >= c.world) continue;
          if (src == c.rank) {
#pragma unroll
            for (int k = 0; k < 4; ++k) u[sj][k] = part[k];
          } else {
            const bf16* sp = slot_ptr(c, c.rank, jo, src, q) + mlc * 32;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int e = lane + 32 * k;
              u[sj][k] = __ldcg(reinterpret_cast<const uint4*>(sp + (e >> 2) * 32 + 8 * (e & 3)));
            }
          }
        }
#pragma unroll
        for (int sj = 0; sj < 4; ++sj) {
          if (s0 + sj >= c.world) continue;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            float f[8];
            unpack8(u[sj][k], f);
#pragma unroll
            for (int i = 0; i < 8; ++i) sum[k][i] += f[i];
          }
        }
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (!live[k]) continue;
        const int e = lane + 32 * k;
        const int ml = mlc + (e >> 2), rv = 8 * (e & 3);
        const int m = tt * kWBN + ml, row = ft * kWBM + 32 * q + rv;
        float hf[8];
        unpack8(hv[k], hf);
#pragma unroll
        for (int i = 0; i < 8; ++i) hf[i] += rbf(sum[k][i]);
        uint4 out;
        pack8(hf, out);
        *reinterpret_cast<uint4*>(a.h + (size_t)m * t.N + row) = out;
        for (int d = 0; d < c.world; ++d)
          if (d != c.rank) *reinterpret_cast<uint4*>(result_ptr(c, d, tile, q) + ml * 32 + rv) = out;
      }
    }
    __syncwarp();  // the staging buffer is refilled by the next chunk
  }
  // publish the quarter: every lane fences its own stores first
  __threadfence_system();
  __syncwarp();
  if (lane == 0) {
    if (!mine) {
      st_release_sys(pflag_ptr(c, owner, jo, c.rank, q), epoch);
    } else {
      for (int d = 0; d < c.world; ++d)
        if (d != c.rank) st_release_sys(rflag_ptr(c, d, tile, q), epoch);
    }
  }
}

// The k-th tile this CTA computes (tiles.. from blockIdx.x in steps of the grid),
// t.tiles past the end.  With the tile exchange, the tiles other ranks own come
// first (their partials are pushed without waiting) and this rank's own tiles
// last, so by the time the owner sums a tile its peers have had the whole first
// part of the schedule to push their partials of it: the owner's epilogue, and
// with it the tensor cores, no longer idle at every owned tile.  Deadlock-free:
// the first part never waits, the second part waits only on it.
template <int EPI>
__device__ __forceinline__ int wide_tile_at(const WideArgs& t, const CommDev& c, int k) {
  const int G = gridDim.x, b = blockIdx.x;
  if (!(EPI == EPI_ROWAR && c.world > 1)) return b + k * G < t.tiles ? b + k * G : t.tiles;
  int seen = 0;
  for (int pass = 0; pass < 2; ++pass)
    for (int tile = b; tile < t.tiles; tile += G)
      if (((tile % c.world) == c.rank) == (pass == 1) && seen++ == k) return tile;
  return t.tiles;
}

template <int EPI>
__global__ void __launch_bounds__(kWThreads, 1) k_wide_gemm(const __grid_constant__ CUtensorMap tw,
                                                            const __grid_constant__ CUtensorMap tx, const WideArgs t,
                                                            const GemvArgs a, const CommDev c) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kWRingBytes);
  uint64_t* empty = full + kWStages;
  uint64_t* accf = empty + kWStages;  // [2] accumulator ready (MMA -> epilogue)
  uint64_t* acce = accf + 2;          // [2] accumulator drained (epilogue -> MMA)
  uint64_t* fin = acce + 2;           // every MMA of the CTA complete
  uint32_t* misc = reinterpret_cast<uint32_t*>(fin + 1);  // tmem base, abort
  volatile uint32_t* abort_flag = misc + 1;
  bf16* stg = reinterpret_cast<bf16*>(smem + kWStageOff);  // [4 warps][32 tokens][32 rows] (exchange)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s_u32(misc)),
                 "r"(kWTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kWStages; ++s) {
      tc_mbar_init(full + s, 1);
      tc_mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc_mbar_init(accf + b, 1);
      tc_mbar_init(acce + b, 4);
    }
    tc_mbar_init(fin, 1);
    misc[1] = 0u;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc[0];
  pdl_launch_dependents();
  if (threadIdx.x == 0) wide_stamp(t, 0);

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      tma_prefetch_map(&tw);
      tma_prefetch_map(&tx);
      pdl_wait();  // the activations come from the previous kernel
      uint32_t it = 0;
      bool ok = true;
      for (int k = 0, tile = wide_tile_at<EPI>(t, c, 0); tile < t.tiles && ok;
           ++k, tile = wide_tile_at<EPI>(t, c, k)) {
        int ft, tt;
        wide_tile(t, tile, ft, tt);
        for (int kb = 0; kb < t.kblocks; ++kb, ++it) {
          const int s = it % kWStages;
          if (it >= (uint32_t)kWStages && !w_wait(empty + s, ((it / kWStages) - 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          unsigned char* st = smem + (size_t)s * kWStageBytes;
          tc_expect_tx(full + s, kWStageBytes);
          tma_load_2d(st, &tw, kb * kTcBK, ft * kWBM, full + s);
          tma_load_2d(st + kWABytes, &tx, kb * kTcBK, tt * kWBN, full + s);
        }
      }
      wide_stamp(t, 6);
      // every copy issued must land before the CTA exits
      const uint32_t first = it > (uint32_t)kWStages ? it - kWStages : 0u;
      for (uint32_t j = first; j < it; ++j) w_wait(full + j % kWStages, (j / kWStages) & 1, nullptr);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t it = 0, ai = 0;
      bool ok = true;
      for (int k = 0, tile = wide_tile_at<EPI>(t, c, 0); tile < t.tiles && ok;
           ++k, tile = wide_tile_at<EPI>(t, c, k), ++ai) {
        const uint32_t b = ai & 1;
        if (ai >= 2 && !w_wait(acce + b, ((ai >> 1) - 1) & 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem + b * kWBN;
        for (int kb = 0; kb < t.kblocks; ++kb, ++it) {
          const int s = it % kWStages;
          if (!w_wait(full + s, (it / kWStages) & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = s_u32(smem + (size_t)s * kWStageBytes);
          const uint32_t sb = sa + kWABytes;
#pragma unroll
          for (int kk = 0; kk < kTcBK / 16; ++kk)
            tc_mma(d, umma_desc_sw128(sa + kk * 32), umma_desc_sw128(sb + kk * 32), kWIdesc,
                   (kb != 0 || kk != 0) ? 1u : 0u);
          tc_commit(empty + s);
        }
        if (ok) tc_commit(accf + b);
      }
      wide_stamp(t, 5);
      tc_commit(fin);  // arrives once every MMA issued above has completed
      w_wait(fin, 0, nullptr);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue warps ----------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int odd = lane & 1;
    pdl_wait();  // the epilogue reads and writes what earlier kernels use
    const bool xchg = EPI == EPI_ROWAR && c.world > 1;
    const uint32_t epoch = xchg ? read_epoch(c) : 0u;
    uint32_t ai = 0;
    for (int k = 0, tile = wide_tile_at<EPI>(t, c, 0); tile < t.tiles;
         ++k, tile = wide_tile_at<EPI>(t, c, k), ++ai) {
      const uint32_t b = ai & 1;
      // warp-uniform: the tcgen05.ld below needs the whole warp
      if (!__all_sync(0xffffffffu, w_wait(accf + b, (ai >> 1) & 1, abort_flag))) break;
      tc_fence_after();
      if (warp == 2 && lane == 0) {
        if (ai == 0) wide_stamp(t, 1);
        // the first owned tile: the tiles other ranks own are done
        if (xchg && tile % c.world == c.rank && (ai == 0 || wide_tile_at<EPI>(t, c, k - 1) % c.world != c.rank))
          wide_stamp(t, 2);
      }
      int ft, tt;
      wide_tile(t, tile, ft, tt);
      const int row0 = (ft * kWBM + 32 * q + lane) & ~1;  // this lane's row pair
      const int g = row0 >> 1;
      const bool live = row0 < t.N;
      float b0 = 0.f, b1 = 0.f;
      if (EPI == EPI_LINEAR && a.bias && live) {
        b0 = ldbf(a.bias + row0);
        b1 = ldbf(a.bias + row0 + 1);
      }
      if (xchg) {
        wide_exchange_tile(c, t, a, tile, ft, tt, q, lane, epoch, tmem + ((uint32_t)(32 * q) << 16) + b * kWBN,
                           acce + b, stg + (warp - 2) * (32 * 32));
        continue;
      }
      if (EPI == EPI_ROWAR && a.addend == nullptr && (t.N & 7) == 0) {
        wide_rowar_tile(t, a, ft, tt, q, lane, tmem + ((uint32_t)(32 * q) << 16) + b * kWBN, acce + b,
                        stg + (warp - 2) * (32 * 32));
        continue;
      }
      // row-parallel: this lane's residual pairs of 16 tokens per 32-token chunk, loaded one
      // chunk ahead (the next chunk's loads are issued before this chunk's stores: the
      // compiler cannot prove the stores do not alias later loads, so loads issued after
      // them would each wait for a round trip)
      uint32_t hv[16];
      if constexpr (EPI == EPI_ROWAR) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = tt * kWBN + 16 * odd + j;
          hv[j] = (live && m < t.M) ? *reinterpret_cast<const uint32_t*>(a.h + (size_t)m * a.N + row0) : 0u;
        }
      }
#pragma unroll 1
      for (int ch = 0; ch < kWBN / 32; ++ch) {
        float v[32];
        tc_ld32(tmem + ((uint32_t)(32 * q) << 16) + b * kWBN + 32 * ch, v);
        if (ch == kWBN / 32 - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) tc_arrive(acce + b);
        }
        const int m0 = tt * kWBN + 32 * ch + 16 * odd;
        if constexpr (EPI == EPI_ROWAR) {
          uint32_t hn[16], ad[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = m0 + j, mn = m + 32;
            const bool ok = live && m < t.M;
            hn[j] = (ch + 1 < kWBN / 32 && live && mn < t.M)
                        ? *reinterpret_cast<const uint32_t*>(a.h + (size_t)mn * a.N + row0) : 0u;
            ad[j] = (ok && a.addend) ? *reinterpret_cast<const uint32_t*>(a.addend + (size_t)m * a.N + row0) : 0u;
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float own = odd ? v[16 + j] : v[j];
            const float other = __shfl_xor_sync(0xffffffffu, odd ? v[j] : v[16 + j], 1);
            const int m = m0 + j;
            if (live && m < t.M) {
              float v0 = odd ? other : own, v1 = odd ? own : other;
              if (a.addend) {
                v0 += __uint_as_float(ad[j] << 16);
                v1 += __uint_as_float(ad[j] & 0xffff0000u);
              }
              *reinterpret_cast<uint32_t*>(a.h + (size_t)m * a.N + row0) =
                  pack2(__uint_as_float(hv[j] << 16) + rbf(v0), __uint_as_float(hv[j] & 0xffff0000u) + rbf(v1));
            }
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) hv[j] = hn[j];
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            // even lane: rows (own, partner) of token j; odd lane: (partner, own) of token 16 + j
            const float own = odd ? v[16 + j] : v[j];
            const float other = __shfl_xor_sync(0xffffffffu, odd ? v[j] : v[16 + j], 1);
            const int m = m0 + j;
            if (live && m < t.M) wide_pair<EPI>(a, g, m, odd ? other : own, odd ? own : other, b0, b1);
          }
        }
      }
    }
    if (warp == 2 && lane == 0) wide_stamp(t, 3);
    if (xchg) {
      // the tiles this CTA computed for other owners: their finished rows -> h
      for (int tile = blockIdx.x; tile < t.tiles; tile += gridDim.x) {
        if (tile % c.world == c.rank) continue;
        int ft, tt;
        wide_tile(t, tile, ft, tt);
        wait_epoch_sys(c, rflag_ptr(c, c.rank, tile, q), epoch);
        const bf16* res = result_ptr(c, c.rank, tile, q);  // [256 tokens][32 rows]
        const int r0 = ft * kWBM + 32 * q;
        // 32 vectors per lane, 8 loads in flight before their stores
        for (int e0 = 0; e0 < kWBN * 4; e0 += 8 * 32) {
          uint4 vv[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) vv[k] = __ldcg(reinterpret_cast<const uint4*>(res + 8 * (e0 + lane + 32 * k)));
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int e = e0 + lane + 32 * k;
            const int m = tt * kWBN + (e >> 2), row = r0 + 8 * (e & 3);
            if (m < t.M && row < t.N) *reinterpret_cast<uint4*>(a.h + (size_t)m * t.N + row) = vv[k];
          }
        }
      }
    }
    if (warp == 2 && lane == 0) wide_stamp(t, 4);
    __syncwarp();
  }

  // ---------------- teardown ----------------
  pdl_wait();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kWTmemCols)
                 : "memory");
  }
  if (threadIdx.x == 0) wide_stamp(t, 7);
  if (EPI == EPI_ROWAR && c.world > 1 && threadIdx.x == 0) {
    // the last CTA advances the comm's call counter (the epoch of the next call)
    const uint32_t epoch = read_epoch(c);
    if (atomicAdd(c.state + kDone, 1u) == gridDim.x - 1) {
      c.state[kDone] = 0u;
      __threadfence();
      c.state[kCalls] = epoch;
    }
  }
}

// ---- host ------------------------------------------------------------------------
struct WidePlan {
  WideArgs t;
  int grid;
  size_t bytes;
};

uint64_t* tc_trace_buffer();  // tc_gemm.cu (jsx_tc_set_trace)

static WidePlan wide_plan(int M, int K, int N, bool norm) {
  WidePlan p;
  p.t.M = M;
  p.t.N = N;
  p.t.K = K;
  p.t.kblocks = (K + kTcBK - 1) / kTcBK;
  p.t.ntt = (M + kWBN - 1) / kWBN;
  p.t.nft = (N + kWBM - 1) / kWBM;
  p.t.tiles = p.t.ntt * p.t.nft;
  p.t.trace = tc_trace_buffer();
  const int sms = sm_count();
  p.grid = p.t.tiles < sms ? p.t.tiles : sms;
  p.bytes = kWOffXn + (norm ? (((size_t)M * K * 2 + 1023) & ~(size_t)1023) : 0);
  return p;
}

CommDev comm_view(jsx_comm* comm);

template <int EPI>
static int wide_run(jsx_comm* comm, GemvArgs ga, void* workspace, size_t workspace_bytes, cudaStream_t s) {
  JSX_REQUIRE(ga.M >= 1, "M=%d", ga.M);
  JSX_REQUIRE(ga.K >= 8 && ga.K % 8 == 0, "K=%d must be a positive multiple of 8", ga.K);
  JSX_REQUIRE(ga.N >= 2 && ga.N % 2 == 0, "N=%d must be even", ga.N);
  JSX_REQUIRE(aligned16(ga.x) && aligned16(ga.w), "activation and weight must be 16-byte aligned");
  JSX_REQUIRE((EPI != EPI_LINEAR || aligned16(ga.y)) && (EPI != EPI_ROWAR || aligned16(ga.h)),
              "output must be 16-byte aligned");
  const WidePlan p = wide_plan(ga.M, ga.K, ga.N, ga.gamma != nullptr);
  JSX_REQUIRE(workspace && aligned16(workspace) && workspace_bytes >= p.bytes,
              "workspace of %zu bytes (16-byte aligned) required", p.bytes);
  CommDev c = {};
  c.world = 1;
  if (EPI == EPI_ROWAR && comm) {
    c = comm_view(comm);
    JSX_REQUIRE(c.world == 1 || c.max_tiles > 0, "the comm has no tile exchange (jsx_comm_create_tiles)");
    JSX_REQUIRE(c.world == 1 || (ga.M <= c.max_tokens && ga.N <= c.hidden), "M=%d N=%d exceed the comm (%d, %d)",
                ga.M, ga.N, c.max_tokens, c.hidden);
    JSX_REQUIRE(c.world == 1 || ga.N % 8 == 0, "N=%d must be a multiple of 8 across ranks", ga.N);
  }
  const void* x = ga.x;
  if (ga.gamma) {
    // RMS-normalised copy of the activations (layers/normalization.py:31-37)
    unsigned char* xn = (unsigned char*)workspace + kWOffXn;
    const int st = jsx_rmsnorm(ga.x, ga.gamma, xn, ga.M, ga.K, ga.eps, s);
    if (st) return st;
    x = xn;
  }
  CUtensorMap tw, tx;
  int st = make_map(&tw, ga.w, ga.N, ga.K, kWBM);
  if (st) return st;
  st = make_map(&tx, x, ga.M, ga.K, kWBN);
  if (st) return st;
  auto kern = k_wide_gemm<EPI>;
  JSX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kWSmem));
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(kWThreads);
  cfg.dynamicSmemBytes = kWSmem;
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (launch_flags() & JSX_LAUNCH_PDL) ? 1 : 0;
  JSX_CUDA(cudaLaunchKernelEx(&cfg, kern, tw, tx, p.t, ga, c));
  return JSX_OK;
}

}  // namespace jsx

using namespace jsx;

extern "C" int jsx_wide_workspace_size(int M, int K, int N, int has_gamma, size_t* bytes) {
  JSX_REQUIRE(bytes && M >= 1 && K >= 8 && N >= 2, "bad arguments");
  *bytes = wide_plan(M, K, N, has_gamma != 0).bytes;
  return JSX_OK;
}

extern "C" int jsx_wide_linear(const void* x, const void* gamma, float eps, const void* w_nk, const void* bias,
                               void* y, int M, int K, int N, void* workspace, size_t workspace_bytes, void* stream) {
  JSX_REQUIRE(x && w_nk && y, "null pointer argument");
  GemvArgs a = {};
  a.x = (const bf16*)x; a.gamma = (const bf16*)gamma; a.eps = eps; a.w = (const bf16*)w_nk;
  a.M = M; a.K = K; a.N = N; a.bias = (const bf16*)bias; a.y = (bf16*)y;
  return wide_run<EPI_LINEAR>(nullptr, a, workspace, workspace_bytes, (cudaStream_t)stream);
}

extern "C" int jsx_wide_qkv_rope_cache(const void* h, const void* ln_gamma, float eps, const void* w_qkv,
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
  return wide_run<EPI_QKV>(nullptr, a, workspace, workspace_bytes, (cudaStream_t)stream);
}

extern "C" int jsx_wide_gate_up_swiglu(const void* h, const void* ln_gamma, float eps, const void* w_gu, void* act,
                                       int M, int K, int I, void* workspace, size_t workspace_bytes, void* stream) {
  JSX_REQUIRE(h && w_gu && act, "null pointer argument");
  GemvArgs a = {};
  a.x = (const bf16*)h; a.gamma = (const bf16*)ln_gamma; a.eps = eps; a.w = (const bf16*)w_gu;
  a.M = M; a.K = K; a.N = 2 * I; a.y = (bf16*)act;
  return wide_run<EPI_SWIGLU>(nullptr, a, workspace, workspace_bytes, (cudaStream_t)stream);
}

extern "C" int jsx_wide_row_linear_allreduce(jsx_comm* comm, const void* x, const void* w_nk, void* h, int M,
                                             int K_local, int N, void* workspace, size_t workspace_bytes,
                                             void* stream) {
  JSX_REQUIRE(x && w_nk && h, "null pointer argument");
  GemvArgs a = {};
  a.x = (const bf16*)x; a.w = (const bf16*)w_nk; a.M = M; a.K = K_local; a.N = N; a.h = (bf16*)h;
  return wide_run<EPI_ROWAR>(comm, a, workspace, workspace_bytes, (cudaStream_t)stream);
}
