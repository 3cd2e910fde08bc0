// MoE experts of one rank (GLM-4.7-Flash, layers/moe.py:194-267).
//
// Per call: N tokens (the normalised hidden states), their top-K expert ids and
// routing weights (jsx_moe_gate).  Each rank computes the experts it owns
// (expert_owner[e] == rank, or every expert without an owner table) for the
// tokens routed to them and returns its routed partial [N][H] in bf16; the
// ranks' partials are summed by the row-parallel all-reduce of the shared
// expert's down projection (jsx_row_linear_allreduce_add), which is where the
// reference's psum("expert") (layers/moe.py:230) happens.
//
//   k_moe_sort      one CTA: stable counting sort of the (token, k) pairs by
//                   owned expert -> per-expert offsets, the pair list, each
//                   pair's slot, and the list of experts with tokens;
//   k_moe_gate_up   grouped GEMV: CTA (active expert, row slice) streams its
//                   slice of the expert's packed gate/up rows once per chunk of
//                   up to 8 of the expert's tokens (gathered into shared
//                   memory) and writes act = bf16(silu(bf16(x Wg)) * bf16(x Wu));
//   k_moe_down      grouped GEMV over the down rows: eo = bf16(act Wd);
//   k_moe_combine   per token, k = 0..K-1 in order over the owned experts:
//                   out = bf16(out + bf16(eo * w_k)) (_topk_local_forward's
//                   bf16 accumulation; experts of other ranks add exactly 0).
#include "common.cuh"
#include "gemv_core.cuh"
#include "launch.cuh"

namespace jsx {

constexpr int kMoeMaxTokens = 32;
constexpr int kMoeMaxK = 8;
constexpr int kMoeMaxE = 256;
constexpr int kMoeChunk = 8;  // tokens per weight pass (the GEMV's M)

struct MoeArgs {
  const bf16* x;           // [N][H]
  const bf16* tk_w;        // [N][K]
  const int32_t* tk_i;     // [N][K]
  const int32_t* owner;    // [E] or null
  int rank;
  int N, K, E, H, I;
  const bf16* w_gu;        // [E][2I][H], rows (gate_j, up_j) interleaved
  const bf16* w_d;         // [E][H][I]
  bf16* out;               // [N][H]
  int32_t* off;            // [E+1]
  int32_t* pairs;          // [N*K] pair ids n*K+k grouped by expert (stable)
  int32_t* slot;           // [N*K] position in pairs, -1 when another rank owns the expert
  int32_t* active;         // [min(E, N*K)] experts with tokens, then -1
  bf16* act;               // [N*K][I]
  bf16* eo;                // [N*K][H]
  int splits;              // CTAs per active expert
};

__global__ void __launch_bounds__(256) k_moe_sort(MoeArgs a) {
  __shared__ int cnt[kMoeMaxE];
  __shared__ int ids[kMoeMaxTokens * kMoeMaxK];
  pdl_wait();
  const int P = a.N * a.K;
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) cnt[e] = 0;
  for (int p = threadIdx.x; p < P; p += blockDim.x) {
    const int e = a.tk_i[p];
    const bool mine = e >= 0 && e < a.E && (a.owner == nullptr || a.owner[e] == a.rank);
    ids[p] = mine ? e : -1;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int p = 0; p < P; ++p)
      if (ids[p] >= 0) ++cnt[ids[p]];
    int run = 0, nact = 0;
    const int amax = a.E < P ? a.E : P;
    for (int e = 0; e < a.E; ++e) {
      a.off[e] = run;
      if (cnt[e] > 0 && nact < amax) a.active[nact++] = e;
      const int c = cnt[e];
      cnt[e] = run;  // cursor
      run += c;
    }
    a.off[a.E] = run;
    for (int i = nact; i < amax; ++i) a.active[i] = -1;
    for (int p = 0; p < P; ++p) {
      const int e = ids[p];
      if (e >= 0) {
        const int s = cnt[e]++;
        a.pairs[s] = p;
        a.slot[p] = s;
      } else {
        a.slot[p] = -1;
      }
    }
  }
  pdl_launch_dependents();
}

// Stage M token rows into shared memory: row m is x[src(m)] (K elements).
template <int M>
__device__ __forceinline__ void stage_rows(const bf16* base, const int32_t* rows, int row_div, int K, bf16* xs,
                                           bool gather) {
  const int nvec = K >> 3;
  uint4* sv = reinterpret_cast<uint4*>(xs);
  for (int i = threadIdx.x; i < M * nvec; i += blockDim.x) {
    const int m = i / nvec, v = i - m * nvec;
    const size_t r = gather ? (size_t)(rows[m] / row_div) : (size_t)m;
    sv[i] = reinterpret_cast<const uint4*>(base + r * K)[v];
  }
  __syncthreads();
}

// One expert, one chunk of M tokens: row pairs [g0, g1) of the expert's weight.
template <int M, int EPI>
__device__ __forceinline__ void moe_chunk(const GemvArgs& ga, int g0, int g1, const bf16* xs) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nvec = ga.K >> 3;
  const uint4* wbase = reinterpret_cast<const uint4*>(ga.w);
  const uint4* xv = reinterpret_cast<const uint4*>(xs);
  for (int g = g0 + warp; g < g1; g += kWarps) {
    const uint4* wv = wbase + (size_t)g * kRows * nvec;
    float acc[kRows][M];
#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
      for (int m = 0; m < M; ++m) acc[r][m] = 0.f;
    Batch bt;
    for (int base = 0; base < nvec; base += 32 * kUnroll) {
      load_batch(bt, wv, nvec, base, lane);
      fma_batch<M>(bt, xv, nvec, base, lane, acc);
    }
#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
      for (int m = 0; m < M; ++m) acc[r][m] = warp_sum(acc[r][m]);
    if constexpr (EPI == EPI_SWIGLU) {
      epi_swiglu<M>(ga, g, acc, lane);
    } else {
      // bf16(act Wd), rows 2g and 2g+1
      if (lane < kRows * M) {
        const int r = lane / M, m = lane - (lane / M) * M;
        ga.y[(size_t)m * ga.N + g * kRows + r] = __float2bfloat16_rn(pick<M>(acc, r, m));
      }
    }
  }
}

template <int EPI>
__global__ void __launch_bounds__(kThreads) k_moe_gemv(MoeArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  bf16* xs = reinterpret_cast<bf16*>(smem_raw);
  pdl_wait();
  const int amax = a.E < a.N * a.K ? a.E : a.N * a.K;
  const int ai = blockIdx.x / a.splits, sp = blockIdx.x - ai * a.splits;
  if (ai >= amax) return;
  const int e = a.active[ai];
  if (e < 0) return;
  const int p0 = a.off[e], cnt = a.off[e + 1] - p0;
  const bool up = EPI == EPI_SWIGLU;
  const int K = up ? a.H : a.I;           // reduction length
  const int Nrows = up ? 2 * a.I : a.H;   // weight rows
  const int npairs = Nrows / kRows;
  const int g0 = (int)((long long)sp * npairs / a.splits), g1 = (int)((long long)(sp + 1) * npairs / a.splits);
  GemvArgs ga = {};
  ga.w = up ? a.w_gu + (size_t)e * 2 * a.I * a.H : a.w_d + (size_t)e * a.H * a.I;
  ga.K = K;
  ga.N = Nrows;
  for (int c0 = 0; c0 < cnt; c0 += kMoeChunk) {
    const int M = cnt - c0 < kMoeChunk ? cnt - c0 : kMoeChunk;
    ga.M = M;
    ga.y = up ? a.act + (size_t)(p0 + c0) * a.I : a.eo + (size_t)(p0 + c0) * a.H;
    __syncthreads();  // the previous chunk's readers of xs are done
#define JSX_MOE_CHUNK(MM)                                                                      \
  {                                                                                            \
    if (up) stage_rows<MM>(a.x, a.pairs + p0 + c0, a.K, K, xs, true);                          \
    else stage_rows<MM>(a.act + (size_t)(p0 + c0) * a.I, nullptr, 1, K, xs, false);           \
    moe_chunk<MM, EPI>(ga, g0, g1, xs);                                                        \
  }
    switch (M) {
      case 1: JSX_MOE_CHUNK(1) break;
      case 2: JSX_MOE_CHUNK(2) break;
      case 3: JSX_MOE_CHUNK(3) break;
      case 4: JSX_MOE_CHUNK(4) break;
      case 5: JSX_MOE_CHUNK(5) break;
      case 6: JSX_MOE_CHUNK(6) break;
      case 7: JSX_MOE_CHUNK(7) break;
      default: JSX_MOE_CHUNK(8) break;
    }
#undef JSX_MOE_CHUNK
  }
  pdl_launch_dependents();
}

__global__ void __launch_bounds__(256) k_moe_combine(MoeArgs a) {
  pdl_wait();
  const int n = blockIdx.x;
  const int hv = a.H >> 3;
  for (int v = threadIdx.x; v < hv; v += blockDim.x) {
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    for (int k = 0; k < a.K; ++k) {
      const int s = a.slot[n * a.K + k];
      if (s < 0) continue;
      const float w = __bfloat162float(a.tk_w[n * a.K + k]);
      float f[8];
      unpack8(reinterpret_cast<const uint4*>(a.eo + (size_t)s * a.H)[v], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = rbf(acc[j] + rbf(f[j] * w));
    }
    uint4 o;
    o.x = pack2(acc[0], acc[1]);
    o.y = pack2(acc[2], acc[3]);
    o.z = pack2(acc[4], acc[5]);
    o.w = pack2(acc[6], acc[7]);
    reinterpret_cast<uint4*>(a.out + (size_t)n * a.H)[v] = o;
  }
  pdl_launch_dependents();
}

struct MoeLayout {
  size_t off, pairs, slot, active, act, eo, bytes;
};

static MoeLayout moe_layout(int N, int K, int E, int H, int I) {
  auto r256 = [](size_t x) { return (x + 255) & ~(size_t)255; };
  MoeLayout L;
  const size_t P = (size_t)N * K;
  L.off = 0;
  L.pairs = r256(L.off + (E + 1) * sizeof(int32_t));
  L.slot = r256(L.pairs + P * sizeof(int32_t));
  L.active = r256(L.slot + P * sizeof(int32_t));
  L.act = r256(L.active + P * sizeof(int32_t));
  L.eo = r256(L.act + P * I * sizeof(bf16));
  L.bytes = r256(L.eo + P * H * sizeof(bf16));
  return L;
}

}  // namespace jsx

using namespace jsx;

extern "C" int jsx_moe_experts_workspace_size(int N, int K, int E, int H, int I, size_t* bytes) {
  JSX_REQUIRE(bytes && N >= 1 && K >= 1 && E >= 1 && H >= 8 && I >= 2, "bad MoE shape");
  *bytes = moe_layout(N, K, E, H, I).bytes;
  return JSX_OK;
}

extern "C" int jsx_moe_experts(const void* x, const void* topk_w, const int32_t* topk_idx,
                               const int32_t* expert_owner, int rank, int N, int K, int E, int H, int I,
                               const void* w_gate_up, const void* w_down, void* out, void* workspace,
                               size_t workspace_bytes, void* stream) {
  JSX_REQUIRE(x && topk_w && topk_idx && w_gate_up && w_down && out, "null pointer argument");
  JSX_REQUIRE(N >= 1 && N <= kMoeMaxTokens, "N=%d outside 1..%d", N, kMoeMaxTokens);
  JSX_REQUIRE(K >= 1 && K <= kMoeMaxK && E >= 1 && E <= kMoeMaxE, "K=%d E=%d", K, E);
  JSX_REQUIRE(H >= 8 && H % 8 == 0 && I >= 8 && I % 8 == 0, "H=%d and I=%d must be multiples of 8", H, I);
  JSX_REQUIRE(aligned16(x) && aligned16(w_gate_up) && aligned16(w_down) && aligned16(out),
              "activations, weights and out must be 16-byte aligned");
  const MoeLayout L = moe_layout(N, K, E, H, I);
  JSX_REQUIRE(workspace && aligned16(workspace) && workspace_bytes >= L.bytes,
              "workspace of %zu bytes required", L.bytes);
  const size_t smem = (size_t)kMoeChunk * (H > I ? H : I) * sizeof(bf16);
  JSX_REQUIRE(smem <= kMaxDynSmem, "H/I too large for the token staging");
  unsigned char* ws = (unsigned char*)workspace;
  MoeArgs a;
  a.x = (const bf16*)x; a.tk_w = (const bf16*)topk_w; a.tk_i = topk_idx; a.owner = expert_owner; a.rank = rank;
  a.N = N; a.K = K; a.E = E; a.H = H; a.I = I;
  a.w_gu = (const bf16*)w_gate_up; a.w_d = (const bf16*)w_down; a.out = (bf16*)out;
  a.off = (int32_t*)(ws + L.off); a.pairs = (int32_t*)(ws + L.pairs); a.slot = (int32_t*)(ws + L.slot);
  a.active = (int32_t*)(ws + L.active); a.act = (bf16*)(ws + L.act); a.eo = (bf16*)(ws + L.eo);
  const int amax = E < N * K ? E : N * K;
  // about two CTAs per SM over the experts that can be active
  int splits = (2 * sm_count() + amax - 1) / amax;
  const int pairs_min = (I < H ? I : H) / kRows;
  if (splits > pairs_min) splits = pairs_min;
  if (splits < 1) splits = 1;
  a.splits = splits;
  cudaStream_t s = (cudaStream_t)stream;
  JSX_CUDA(launch_kernel(k_moe_sort, dim3(1), dim3(256), 0, s, a));
  auto kgu = k_moe_gemv<EPI_SWIGLU>;
  auto kd = k_moe_gemv<EPI_LINEAR>;
  JSX_CUDA(cudaFuncSetAttribute(kgu, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  JSX_CUDA(cudaFuncSetAttribute(kd, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  JSX_CUDA(launch_kernel(kgu, dim3(amax * splits), dim3(kThreads), smem, s, a));
  JSX_CUDA(launch_kernel(kd, dim3(amax * splits), dim3(kThreads), smem, s, a));
  JSX_CUDA(launch_kernel(k_moe_combine, dim3(N), dim3(256), 0, s, a));
  return JSX_OK;
}
