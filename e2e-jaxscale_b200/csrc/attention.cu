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

constexpr int kChunk = 64;  // cache rows per split
constexpr int kSub = kChunk / 32;  // rows per lane in the score phase
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
  float* part;     // [B*nkv][splits][split_stride]: acc [G][hd], then m [G], l [G] (padded)
  uint32_t* cnt;   // [B*nkv], zero on entry, left zero
};

// floats per split record: the accumulator tile, then (m, l) per head, padded so
// every record starts on a 16-byte boundary (float4 reads in the combine)
__host__ __device__ __forceinline__ int split_stride(int G, int hd) {
  return G * hd + ((2 * G + 3) & ~3);
}

__global__ void __launch_bounds__(kAttnThreads) k_attn_decode(AttnArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int G = a.nq / a.nkv;
  const int hd = a.hd, hw = hd >> 1;  // head dim in 4-byte words
  const int stride = split_stride(G, hd);
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
  float* part = a.part + ((size_t)bk * a.splits + s) * stride;

  if (n > 0) {
    const bf16* qg = a.q + ((size_t)b * a.nq + (size_t)kvh * G) * hd;
    for (int i = tid; i < G * hd; i += kAttnThreads) qs[i] = __bfloat162float(qg[i]);
    const size_t row_stride = (size_t)a.nkv * hd;  // elements between consecutive cache rows
    const bf16* kb = a.kc + ((size_t)b * a.max_seq + p0) * row_stride + (size_t)kvh * hd;
    const bf16* vb = a.vc + ((size_t)b * a.max_seq + p0) * row_stride + (size_t)kvh * hd;
    const int hq = hd >> 3;  // 16-byte vectors per row
    for (int i = tid; i < n * hq; i += kAttnThreads) {
      const int r = i / hq, c = i - (i / hq) * hq;
      const uint4 kv = reinterpret_cast<const uint4*>(kb + (size_t)r * row_stride)[c];
      const uint4 vv = reinterpret_cast<const uint4*>(vb + (size_t)r * row_stride)[c];
      uint32_t* kd = ks + r * (hw + 1) + 4 * c;
      kd[0] = kv.x; kd[1] = kv.y; kd[2] = kv.z; kd[3] = kv.w;
      reinterpret_cast<uint4*>(vs + r * hw)[c] = vv;
    }
    __syncthreads();

    // scores: lane handles rows lane + 32 j; q is a broadcast read
    for (int g = warp; g < G; g += kAttnWarps) {
      const float* qr = qs + g * hd;
      float sc[kSub];
#pragma unroll
      for (int j = 0; j < kSub; ++j) {
        const int p = lane + 32 * j;
        sc[j] = -INFINITY;
        if (p < n) {
          const uint32_t* kr = ks + p * (hw + 1);
          float dot = 0.f;
          for (int w = 0; w < hw; ++w) {
            const uint32_t kw = kr[w];
            dot = fmaf(qr[2 * w], bf_lo(kw), dot);
            dot = fmaf(qr[2 * w + 1], bf_hi(kw), dot);
          }
          sc[j] = dot * a.scale;
        }
      }
      float m = sc[0];
#pragma unroll
      for (int j = 1; j < kSub; ++j) m = fmaxf(m, sc[j]);
      m = warp_max(m);
      float l = 0.f;
#pragma unroll
      for (int j = 0; j < kSub; ++j) {
        const float e = (lane + 32 * j < n) ? expf(sc[j] - m) : 0.f;
        ps[g * kChunk + lane + 32 * j] = e;
        l += e;
      }
      l = warp_sum(l);
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

  // Combine the splits holding rows [0, cur]: weights w_t[g] = exp(m_t - M) / L
  // are formed once in shared memory (the staging buffers are free now), then
  // every output element is a short dot product over the splits.
  const int used = (cur + kChunk) / kChunk;
  const float* pb = a.part + (size_t)bk * a.splits * stride;
  float* wm = reinterpret_cast<float*>(ks);  // [used][G] m, then weights
  float* wl = wm + a.splits * G;             // [used][G] l
  float* Mg = wl + a.splits * G;             // [G]
  float* Lg = Mg + G;                        // [G]
  for (int i = tid; i < used * G; i += kAttnThreads) {
    const int t = i / G, g = i - (i / G) * G;
    wm[i] = __ldcg(pb + (size_t)t * stride + G * hd + g);
    wl[i] = __ldcg(pb + (size_t)t * stride + G * hd + G + g);
  }
  __syncthreads();
  for (int g = tid; g < G; g += kAttnThreads) {
    float M = -INFINITY;
    for (int t = 0; t < used; ++t) M = fmaxf(M, wm[t * G + g]);
    float L = 0.f;
    for (int t = 0; t < used; ++t) L = fmaf(wl[t * G + g], expf(wm[t * G + g] - M), L);
    Mg[g] = M;
    Lg[g] = L;
  }
  __syncthreads();
  for (int i = tid; i < used * G; i += kAttnThreads) {
    const int g = i - (i / G) * G;
    wm[i] = expf(wm[i] - Mg[g]) / Lg[g];
  }
  __syncthreads();
  bf16* ob = a.out + ((size_t)b * a.nq + (size_t)kvh * G) * hd;
  const int nv = (G * hd) >> 2;
  for (int i = tid; i < nv; i += kAttnThreads) {
    const int e = i << 2, g = e / hd;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
    for (int t = 0; t < used; ++t) {
      const float w = wm[t * G + g];
      const float4 v = __ldcg(reinterpret_cast<const float4*>(pb + (size_t)t * stride + e));
      o.x = fmaf(v.x, w, o.x);
      o.y = fmaf(v.y, w, o.y);
      o.z = fmaf(v.z, w, o.z);
      o.w = fmaf(v.w, w, o.w);
    }
    uint2 packed;
    packed.x = pack2(o.x, o.y);
    packed.y = pack2(o.z, o.w);
    *reinterpret_cast<uint2*>(ob + e) = packed;
  }
  if (tid == 0) a.cnt[bk] = 0u;
}

// workspace: 256-byte header, then the per-(b, kvh) counters padded to 256 bytes, then the partials
static size_t attn_counter_bytes(int B, int nkv) {
  return 256 + (((size_t)B * nkv * sizeof(uint32_t) + 255) & ~(size_t)255);
}

static size_t attn_smem(int G, int hd, int splits) {
  const int hw = hd / 2;
  const size_t stage = (size_t)kChunk * (hw + 1) * 4 + (size_t)kChunk * hw * 4;
  const size_t combine = ((size_t)2 * splits * G + 2 * G) * 4;
  return (size_t)G * hd * 4 + (size_t)G * kChunk * 4 + (stage > combine ? stage : combine);
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
  *bytes = attn_counter_bytes(B, nkv) + (size_t)B * nkv * splits * split_stride(G, head_dim) * sizeof(float);
  return JSX_OK;
}

extern "C" int jsx_attn_decode(const void* q, const void* k_cache, const void* v_cache, void* out,
                               const int32_t* positions, int B, int nq, int nkv, int head_dim,
                               int max_seq, float scale, void* workspace, size_t workspace_bytes,
                               void* stream) {
  JSX_REQUIRE(q && k_cache && v_cache && out && positions, "null pointer argument");
  JSX_REQUIRE(B >= 1 && nq >= 1 && nkv >= 1 && nq % nkv == 0, "bad heads nq=%d nkv=%d", nq, nkv);
  JSX_REQUIRE(head_dim >= 8 && head_dim % 8 == 0 && head_dim <= 512, "head_dim=%d must be a multiple of 8",
              head_dim);
  JSX_REQUIRE(max_seq >= 1, "max_seq=%d", max_seq);
  JSX_REQUIRE(aligned16(k_cache) && aligned16(v_cache) && aligned16(out),
              "caches and out must be 16-byte aligned");
  const int G = nq / nkv;
  size_t need = 0;
  jsx_attn_decode_workspace_size(B, nq, nkv, head_dim, max_seq, &need);
  JSX_REQUIRE(workspace && workspace_bytes >= need && aligned16(workspace),
              "workspace of %zu bytes (16-byte aligned) required, got %zu", need, workspace_bytes);
  const int splits = (max_seq + kChunk - 1) / kChunk;
  const size_t smem = attn_smem(G, head_dim, splits);
  JSX_REQUIRE(smem <= 200 * 1024, "attention tile too large (G=%d hd=%d)", G, head_dim);
  AttnArgs a;
  a.q = (const bf16*)q; a.kc = (const bf16*)k_cache; a.vc = (const bf16*)v_cache;
  a.out = (bf16*)out; a.pos = positions; a.B = B; a.nq = nq; a.nkv = nkv; a.hd = head_dim;
  a.max_seq = max_seq; a.splits = splits; a.scale = scale;
  a.cnt = (uint32_t*)((char*)workspace + 256);
  a.part = (float*)((char*)workspace + attn_counter_bytes(B, nkv));
  auto kern = k_attn_decode;
  JSX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  JSX_CUDA(launch_kernel(kern, dim3(a.splits, B * nkv), dim3(kAttnThreads), smem,
                         (cudaStream_t)stream, a));
  return JSX_OK;
}
