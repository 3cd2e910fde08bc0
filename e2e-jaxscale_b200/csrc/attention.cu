// Decode attention over the static KV cache (GQA), split over the context.
//
// Reference: layers/attention.py:136-153 calls jax.nn.dot_product_attention
// over the WHOLE max_cache_len cache with the additive decode mask of
// runner.py:49-63 (0 for rows <= cur_pos, -1e9 above).  A masked row's
// exp(-1e9 - max) is exactly 0 in fp32, so reading only rows [0, cur_pos]
// computes the same function; this kernel never touches the masked rows.
//
// Grid: (split, b * nkv + kvh).  Each CTA stages kChunk cache rows of one KV
// head in shared memory and serves all G = nq/nkv query heads of the group
// from that single read (GQA reuse).  Scores are fp32 (q.k of bf16 inputs,
// then * scale, as in the reference), softmax is fp32 with a split-local max;
// the last CTA of each (b, kvh) merges the splits (flash-decoding combine).
// Probabilities stay fp32 up to the P.V sum (the reference rounds them to bf16
// first); the output is rounded to bf16 once.
#include <math.h>

#include "common.cuh"
#include "launch.cuh"

namespace jsx {

constexpr int kChunk = 32;  // cache rows per split (one per lane in the score phase)
constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = kAttnThreads / 32;

struct AttnArgs {
  const bf16* q;   // [B][nq][hd]
  const bf16* kc;  // [B][max_seq][nkv][hd]
  const bf16* vc;
  bf16* out;       // [B][nq*hd]
  const int32_t* pos;
  int B, nq, nkv, hd, max_seq, splits;
  float scale;
  float* part;     // [B*nkv][splits][G][hd + 2]  (acc, then m, l per head)
  uint32_t* cnt;   // [B*nkv], zero on entry, left zero
};

__global__ void __launch_bounds__(kAttnThreads) k_attn_decode(AttnArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int G = a.nq / a.nkv;
  const int hd = a.hd, hw = hd >> 1;  // head dim in 4-byte words
  float* qs = reinterpret_cast<float*>(smem_raw);                  // [G][hd]
  float* ps = qs + G * hd;                                          // [G][kChunk]
  uint32_t* ks = reinterpret_cast<uint32_t*>(ps + G * kChunk);      // [kChunk][hw+1] (padded)
  uint32_t* vs = ks + kChunk * (hw + 1);                            // [kChunk][hw]
  __shared__ bool is_last;

  const int s = blockIdx.x, bk = blockIdx.y;
  const int b = bk / a.nkv, kvh = bk - (bk / a.nkv) * a.nkv;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  pdl_wait();
  pdl_launch_dependents();

  int cur = a.pos[b];
  if (cur > a.max_seq - 1) cur = a.max_seq - 1;
  if (cur < 0) cur = 0;
  const int p0 = s * kChunk;
  int n = cur + 1 - p0;
  if (n > kChunk) n = kChunk;
  float* part = a.part + ((size_t)bk * a.splits + s) * G * (hd + 2);

  if (n > 0) {
    const bf16* qg = a.q + ((size_t)b * a.nq + (size_t)kvh * G) * hd;
    for (int i = tid; i < G * hd; i += kAttnThreads) qs[i] = __bfloat162float(qg[i]);
    const size_t row_stride = (size_t)a.nkv * hd;  // elements between consecutive cache rows
    const bf16* kb = a.kc + ((size_t)b * a.max_seq + p0) * row_stride + (size_t)kvh * hd;
    const bf16* vb = a.vc + ((size_t)b * a.max_seq + p0) * row_stride + (size_t)kvh * hd;
    for (int i = tid; i < n * hw; i += kAttnThreads) {
      const int r = i / hw, w = i - (i / hw) * hw;
      ks[r * (hw + 1) + w] = reinterpret_cast<const uint32_t*>(kb + (size_t)r * row_stride)[w];
      vs[r * hw + w] = reinterpret_cast<const uint32_t*>(vb + (size_t)r * row_stride)[w];
    }
    __syncthreads();

    for (int g = warp; g < G; g += kAttnWarps) {
      float sc = -INFINITY;
      if (lane < n) {
        const uint32_t* kr = ks + lane * (hw + 1);
        const float* qr = qs + g * hd;
        float dot = 0.f;
        for (int w = 0; w < hw; ++w) {
          const uint32_t kw = kr[w];
          dot = fmaf(qr[2 * w], bf_lo(kw), dot);
          dot = fmaf(qr[2 * w + 1], bf_hi(kw), dot);
        }
        sc = dot * a.scale;
      }
      const float m = warp_max(sc);
      const float e = (lane < n) ? expf(sc - m) : 0.f;
      const float l = warp_sum(e);
      ps[g * kChunk + lane] = e;
      if (lane == 0) {
        part[G * hd + g] = m;
        part[G * hd + G + g] = l;
      }
    }
    __syncthreads();
    for (int i = tid; i < G * hw; i += kAttnThreads) {
      const int g = i / hw, w = i - (i / hw) * hw;
      float a0 = 0.f, a1 = 0.f;
      const float* pg = ps + g * kChunk;
      for (int p = 0; p < n; ++p) {
        const uint32_t vw = vs[p * hw + w];
        a0 = fmaf(pg[p], bf_lo(vw), a0);
        a1 = fmaf(pg[p], bf_hi(vw), a1);
      }
      part[g * hd + 2 * w] = a0;
      part[g * hd + 2 * w + 1] = a1;
    }
  }

  __threadfence();
  __syncthreads();
  if (tid == 0) is_last = atomicAdd(a.cnt + bk, 1u) == (uint32_t)(a.splits - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();

  const int used = (cur + kChunk) / kChunk;  // splits holding rows [0, cur]
  const float* pb = a.part + (size_t)bk * a.splits * G * (hd + 2);
  bf16* ob = a.out + ((size_t)b * a.nq + (size_t)kvh * G) * hd;
  for (int i = tid; i < G * hd; i += kAttnThreads) {
    const int g = i / hd, d = i - (i / hd) * hd;
    float M = -INFINITY;
    for (int t = 0; t < used; ++t) M = fmaxf(M, __ldcg(pb + (size_t)t * G * (hd + 2) + G * hd + g));
    float L = 0.f, O = 0.f;
    for (int t = 0; t < used; ++t) {
      const float* pt = pb + (size_t)t * G * (hd + 2);
      const float w = expf(__ldcg(pt + G * hd + g) - M);
      L = fmaf(__ldcg(pt + G * hd + G + g), w, L);
      O = fmaf(__ldcg(pt + g * hd + d), w, O);
    }
    ob[g * hd + d] = __float2bfloat16_rn(O / L);
  }
  if (tid == 0) a.cnt[bk] = 0u;
}

// workspace: 256-byte header, then the per-(b, kvh) counters padded to 256 bytes, then the partials
static size_t attn_counter_bytes(int B, int nkv) {
  return 256 + (((size_t)B * nkv * sizeof(uint32_t) + 255) & ~(size_t)255);
}

static size_t attn_smem(int G, int hd) {
  const int hw = hd / 2;
  return (size_t)G * hd * 4 + (size_t)G * kChunk * 4 + (size_t)kChunk * (hw + 1) * 4 +
         (size_t)kChunk * hw * 4;
}

}  // namespace jsx

using namespace jsx;

extern "C" int jsx_attn_decode_workspace_size(int B, int nq, int nkv, int head_dim, int max_seq,
                                              size_t* bytes) {
  JSX_REQUIRE(bytes && B >= 1 && nq >= 1 && nkv >= 1 && nq % nkv == 0 && head_dim >= 2 &&
                  max_seq >= 1,
              "bad attention shape");
  const int G = nq / nkv;
  const int splits = (max_seq + kChunk - 1) / kChunk;
  *bytes = attn_counter_bytes(B, nkv) + (size_t)B * nkv * splits * G * (head_dim + 2) * sizeof(float);
  return JSX_OK;
}

extern "C" int jsx_attn_decode(const void* q, const void* k_cache, const void* v_cache, void* out,
                               const int32_t* positions, int B, int nq, int nkv, int head_dim,
                               int max_seq, float scale, void* workspace, size_t workspace_bytes,
                               void* stream) {
  JSX_REQUIRE(q && k_cache && v_cache && out && positions, "null pointer argument");
  JSX_REQUIRE(B >= 1 && nq >= 1 && nkv >= 1 && nq % nkv == 0, "bad heads nq=%d nkv=%d", nq, nkv);
  JSX_REQUIRE(head_dim >= 2 && head_dim % 2 == 0 && head_dim <= 512, "head_dim=%d", head_dim);
  JSX_REQUIRE(max_seq >= 1, "max_seq=%d", max_seq);
  JSX_REQUIRE(aligned4(q) && aligned4(k_cache) && aligned4(v_cache) && aligned4(out),
              "q/k/v/out must be 4-byte aligned");
  const int G = nq / nkv;
  size_t need = 0;
  jsx_attn_decode_workspace_size(B, nq, nkv, head_dim, max_seq, &need);
  JSX_REQUIRE(workspace && workspace_bytes >= need && aligned16(workspace),
              "workspace of %zu bytes (16-byte aligned) required, got %zu", need, workspace_bytes);
  const size_t smem = attn_smem(G, head_dim);
  JSX_REQUIRE(smem <= 200 * 1024, "attention tile too large (G=%d hd=%d)", G, head_dim);
  AttnArgs a;
  a.q = (const bf16*)q; a.kc = (const bf16*)k_cache; a.vc = (const bf16*)v_cache;
  a.out = (bf16*)out; a.pos = positions; a.B = B; a.nq = nq; a.nkv = nkv; a.hd = head_dim;
  a.max_seq = max_seq; a.splits = (max_seq + kChunk - 1) / kChunk; a.scale = scale;
  a.cnt = (uint32_t*)((char*)workspace + 256);
  a.part = (float*)((char*)workspace + attn_counter_bytes(B, nkv));
  auto kern = k_attn_decode;
  JSX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  JSX_CUDA(launch_kernel(kern, dim3(a.splits, B * nkv), dim3(kAttnThreads), smem,
                         (cudaStream_t)stream, a));
  return JSX_OK;
}
