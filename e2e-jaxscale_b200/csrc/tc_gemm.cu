// Tensor-core decode projections for 1..32 tokens (batch > 8): tcgen05 + TMA.
//
// At batch 32 a weight element feeds 64 flops; the CUDA-core GEMV would be
// compute bound (~8x the HBM time), so these projections run on the 5th-gen
// tensor cores.  Shapes are "skinny": D[128 weight rows, 32 tokens] per tile,
// the weight tile is the MMA's A operand (M = 128) and the token activations
// the B operand (N = 32, zero-filled by TMA beyond the real token count), both
// K-major bf16 with the 128-byte swizzle, fp32 accumulation in TMEM.
//
//   k_tc_gemm       one CTA per (128-row tile, K split): warp 0 / lane 0 loads
//                   the A (16 KB) and B (4 KB) boxes of each 64-wide K block
//                   with cp.async.bulk.tensor into a 4-stage ring; warp 1 /
//                   lane 0 issues 4 tcgen05.mma (K = 16 each) per stage and
//                   hands the stage back with tcgen05.commit; the 4 warps then
//                   read their 32 TMEM lanes (tcgen05.ld 32x32b.x32 = one weight
//                   row x 32 tokens per thread) and store fp32 split partials.
//   k_tc_rows       sums the split partials of each row pair in split order and
//                   runs the same pair epilogues as the GEMV kernels (bias,
//                   RoPE + KV write, SwiGLU, residual + tensor-parallel
//                   all-reduce, LM-head argmax).
//
// No multicast anywhere.  Every mbarrier wait is time-bounded; on a timeout the
// kernel sets its error word (jsx_device_error), drains its own copies and MMAs
// (bounded) and frees its TMEM before returning.
#include <cuda.h>
#include <stdio.h>
#include <stdlib.h>

#include <mutex>

#include "comm.cuh"
#include "common.cuh"
#include "gemv_core.cuh"
#include "launch.cuh"

namespace jsx {

constexpr int kTcBM = 128;  // weight rows per tile (MMA M)
constexpr int kTcBN = 32;   // tokens per tile (MMA N)
constexpr int kTcBK = 64;   // K per stage: one 128-byte swizzle row of bf16
constexpr int kTcStages = 4;
constexpr int kTcThreads = 128;
constexpr int kTcMaxM = 32;
constexpr uint32_t kTcABytes = kTcBM * kTcBK * 2;
constexpr uint32_t kTcBBytes = kTcBN * kTcBK * 2;
constexpr uint32_t kTcStageBytes = kTcABytes + kTcBBytes;
constexpr size_t kTcSmem = (size_t)kTcStages * kTcStageBytes + 1024 /* align */ + 256 /* barriers */;
constexpr long long kTcWaitCycles = 4000000000ll;  // ~2 s at the 1965 MHz max clock

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
  float* part;  // [splits][M][N]
  int M, N, K, kblocks, splits, tiles;
};

__device__ __forceinline__ uint32_t s_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void tc_mbar_init(uint64_t* b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(s_u32(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void tc_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(s_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool tc_try_wait(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(s_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait; false (and the error word set) on timeout.
__device__ __forceinline__ bool tc_wait(uint64_t* b, uint32_t parity) {
  if (tc_try_wait(b, parity)) return true;
  const long long t0 = clock64();
  for (uint32_t it = 1;; ++it) {
    if (tc_try_wait(b, parity)) return true;
    if ((it & 63u) == 0 && clock64() - t0 > kTcWaitCycles) {
      atomicOr(&g_tc_error, 1u);
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(s_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(s_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor of a K-major, 128-byte-swizzled operand tile
// (8-row swizzle atoms of 1024 bytes stacked along the M/N dimension):
// start address, leading byte offset 16 B (unused with this swizzle), stride
// byte offset 1024 B, descriptor version 1, layout type 2 (128-byte swizzle).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)(16u >> 4) << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor of kind::f16: fp32 accumulate, bf16 A and B, both
// K-major, N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t kTcIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTcBN >> 3) << 17) |
                              ((uint32_t)(kTcBM >> 4) << 24);

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(kTcIdesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(s_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__global__ void __launch_bounds__(kTcThreads, 2) k_tc_gemm(const __grid_constant__ CUtensorMap tw,
                                                           const __grid_constant__ CUtensorMap tx, TcArgs a) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kTcStages * kTcStageBytes);
  uint64_t* empty = full + kTcStages;
  uint64_t* accf = empty + kTcStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accf + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x % a.tiles, split = blockIdx.x / a.tiles;
  const int kb0 = (int)((long long)split * a.kblocks / a.splits);
  const int kb1 = (int)((long long)(split + 1) * a.kblocks / a.splits);
  const int nkb = kb1 - kb0;
  const int n0 = tile * kTcBM;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s_u32(tmem_slot)),
                 "r"(32)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x == 32) {
    for (int s = 0; s < kTcStages; ++s) {
      tc_mbar_init(full + s, 1);
      tc_mbar_init(empty + s, 1);
    }
    tc_mbar_init(accf, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---- TMA producer ----
    int i = 0;
    for (; i < nkb; ++i) {
      const int s = i % kTcStages;
      if (i >= kTcStages && !tc_wait(empty + s, ((i / kTcStages) - 1) & 1)) break;
      unsigned char* st = smem + (size_t)s * kTcStageBytes;
      tc_expect_tx(full + s, kTcStageBytes);
      tma_load_2d(st, &tw, (kb0 + i) * kTcBK, n0, full + s);
      tma_load_2d(st + kTcABytes, &tx, (kb0 + i) * kTcBK, 0, full + s);
    }
    // drain: the last loads issued must land before the CTA can exit
    const int first = i > kTcStages ? i - kTcStages : 0;
    for (int j = first; j < i; ++j) tc_wait(full + j % kTcStages, (j / kTcStages) & 1);
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    for (int i = 0; i < nkb; ++i) {
      const int s = i % kTcStages;
      if (!tc_wait(full + s, (i / kTcStages) & 1)) break;
      tc_fence_after();
      const uint32_t sa = s_u32(smem + (size_t)s * kTcStageBytes);
      const uint32_t sb = sa + kTcABytes;
#pragma unroll
      for (int kk = 0; kk < kTcBK / 16; ++kk)
        tc_mma(tmem, umma_desc_sw128(sa + kk * 32), umma_desc_sw128(sb + kk * 32), (i | kk) != 0 ? 1u : 0u);
      tc_commit(empty + s);
    }
    tc_commit(accf);  // fires when every MMA issued above has completed
  }
  __syncwarp();

  // ---- epilogue: thread = one weight row, 32 token columns ----
  const bool ok = tc_wait(accf, 0);
  tc_fence_after();
  float v[32];
  tc_ld32(tmem + ((uint32_t)(warp * 32) << 16), v);
  const int row = n0 + warp * 32 + lane;
  if (ok && row < a.N) {
    float* dst = a.part + (size_t)split * a.M * a.N + row;
#pragma unroll
    for (int t = 0; t < 32; ++t)
      if (t < a.M) dst[(size_t)t * a.N] = v[t];
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(32) : "memory");
  }
}

// ---- row-pair epilogue over the split partials ----------------------------
struct TcRowArgs {
  GemvArgs ga;        // epilogue fields (bias, q/k/v/cache/rope, h, act, logits, keys ...)
  const float* part;  // [splits][M][N]
  int splits;
};

template <int EPI>
__global__ void __launch_bounds__(256) k_tc_rows(TcRowArgs r, CommDev c) {
  const GemvArgs& a = r.ga;
  __shared__ unsigned long long best_s[kTcMaxM];
  __shared__ bool is_last;
  const int M = a.M, NB = a.N >> 1;
  const int p0 = (int)((long long)blockIdx.x * NB / gridDim.x);
  const int p1 = (int)((long long)(blockIdx.x + 1) * NB / gridDim.x);
  const bool multi = (EPI == EPI_ROWAR || EPI == EPI_LMHEAD) && c.world > 1;
  uint32_t epoch = 0;
  int par = 0;
  if (EPI == EPI_ROWAR && multi) {
    epoch = read_epoch(c);
    par = epoch & 1;
  }
  if (EPI == EPI_LMHEAD && threadIdx.x < kTcMaxM) best_s[threadIdx.x] = 0ull;
  __syncthreads();
  const size_t plane = (size_t)M * a.N;
  for (int e = threadIdx.x; e < (p1 - p0) * M; e += blockDim.x) {
    const int m = e / (p1 - p0), g = p0 + (e - m * (p1 - p0));
    const float* src = r.part + (size_t)m * a.N + 2 * g;
    float v0 = 0.f, v1 = 0.f;
    for (int s = 0; s < r.splits; ++s) {
      const float2 t = *reinterpret_cast<const float2*>(src + s * plane);
      v0 += t.x;
      v1 += t.y;
    }
    const unsigned long long k = epi_pair<EPI>(a, c, multi, par, g, m, v0, v1);
    if (EPI == EPI_LMHEAD) atomicMax(best_s + m, k);
  }

  if constexpr (EPI == EPI_ROWAR) {
    if (multi) {
      __threadfence_system();
      __syncthreads();
      if (threadIdx.x < c.world) st_release_sys(flag_ptr(c, threadIdx.x, blockIdx.x, c.rank), epoch);
      if (threadIdx.x < c.world) wait_flag(c, blockIdx.x, threadIdx.x, epoch);
      __syncthreads();
      const int rows = 2 * (p1 - p0);
      for (int e = threadIdx.x; e < rows * M; e += blockDim.x) {
        const int m = e / rows, row = 2 * p0 + (e - (e / rows) * rows);
        float sum = 0.f;
        for (int src = 0; src < c.world; ++src) sum += __ldcg(data_ptr(c, c.rank, par, src, m) + row);
        bf16* hp = a.h + (size_t)m * a.N + row;
        *hp = __float2bfloat16_rn(__bfloat162float(*hp) + rbf(sum));
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
    __syncthreads();
    if (threadIdx.x < M && best_s[threadIdx.x]) atomicMax(a.keys + threadIdx.x, best_s[threadIdx.x]);
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) is_last = atomicAdd(a.done, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    __shared__ unsigned long long fin[kTcMaxM];
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

// ---- host ------------------------------------------------------------------------
typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static int get_encoder(PFN_encodeTiled* out) {
  static PFN_encodeTiled fn = nullptr;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    JSX_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    JSX_REQUIRE(p != nullptr && q == cudaDriverEntryPointSuccess, "cuTensorMapEncodeTiled unavailable");
    fn = (PFN_encodeTiled)p;
  }
  *out = fn;
  return JSX_OK;
}

// 2-D bf16 tensor map over a row-major [rows][K] matrix, box [box_rows][64],
// 128-byte swizzle, out-of-range elements read as zero.
static int make_map(CUtensorMap* map, const void* base, int rows, int K, int box_rows) {
  PFN_encodeTiled enc;
  int st = get_encoder(&enc);
  if (st) return st;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {(cuuint32_t)kTcBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  JSX_REQUIRE(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return JSX_OK;
}

struct TcPlan {
  int tiles, kblocks, splits;
  size_t xn_off, part_off, bytes;
};

// K splits: about 4 CTAs per B200 SM (148 SMs, 2 resident CTAs each: two
// waves), at least 4 K blocks per split.  The plan depends only on the shape,
// so the workspace size and the summation order are the same on every device.
constexpr int kTcTargetCtas = 4 * 148;
static TcPlan tc_plan(int M, int K, int N) {
  TcPlan p;
  p.tiles = (N + kTcBM - 1) / kTcBM;
  p.kblocks = (K + kTcBK - 1) / kTcBK;
  const int target = kTcTargetCtas;
  int splits = (target + p.tiles - 1) / p.tiles;
  int cap = p.kblocks / 4;
  if (cap < 1) cap = 1;
  if (splits > cap) splits = cap;
  if (splits < 1) splits = 1;
  p.splits = splits;
  p.xn_off = 1024;
  p.part_off = p.xn_off + (((size_t)kTcMaxM * K * 2 + 1023) & ~(size_t)1023);
  p.bytes = p.part_off + (size_t)splits * M * N * sizeof(float);
  return p;
}

CommDev comm_view(jsx_comm* comm);

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
  // activations: RMS-normalised copy when a gain is given (layers/normalization.py:31-37)
  const void* x = ga.x;
  if (ga.gamma) {
    const int st = jsx_rmsnorm(ga.x, ga.gamma, ws + p.xn_off, ga.M, ga.K, ga.eps, s);
    if (st) return st;
    x = ws + p.xn_off;
  }
  CUtensorMap tw, tx;
  int st = make_map(&tw, ga.w, ga.N, ga.K, kTcBM);
  if (st) return st;
  st = make_map(&tx, x, ga.M, ga.K, kTcBN);
  if (st) return st;
  TcArgs ta;
  ta.part = (float*)(ws + p.part_off);
  ta.M = ga.M; ta.N = ga.N; ta.K = ga.K; ta.kblocks = p.kblocks; ta.splits = p.splits; ta.tiles = p.tiles;
  JSX_CUDA(cudaFuncSetAttribute(k_tc_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem));
  k_tc_gemm<<<p.tiles * p.splits, kTcThreads, kTcSmem, s>>>(tw, tx, ta);
  JSX_LAUNCHED("k_tc_gemm");
  TcRowArgs ra;
  ra.ga = ga;
  ra.part = ta.part;
  ra.splits = p.splits;
  int grid = 2 * sm_count();
  if (EPI == EPI_ROWAR && grid > kMaxCtas) grid = kMaxCtas;
  if (grid > ga.N / 2) grid = ga.N / 2;
  k_tc_rows<EPI><<<grid, 256, 0, s>>>(ra, c);
  JSX_LAUNCHED("k_tc_rows");
  return JSX_OK;
}

}  // namespace jsx

using namespace jsx;

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
  a.done = (uint32_t*)workspace;                                    // header: done counter
  a.keys = (unsigned long long*)((char*)workspace + 256);          // then M argmax keys
  a.ids = ids_out;
  return tc_run<EPI_LMHEAD>(comm, a, workspace, workspace_bytes, (cudaStream_t)stream);
}
