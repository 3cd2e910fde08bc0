// Decode attention over the static KV cache (GQA), split over the context.
//
// Reference: layers/attention.py:136-153 calls jax.nn.dot_product_attention
// over the WHOLE max_cache_len cache with the additive decode mask of
// runner.py:49-63 (0 for rows <= cur_pos, -1e9 above).  A masked row's
// exp(-1e9 - max) is exactly 0 in fp32, so reading only rows [0, cur_pos]
// computes the same function; this kernel never touches the masked rows.
//
// Grid: (split, item group).  Each CTA stages kChunk cache rows of one KV head
// in shared memory and serves the query heads of its group from that single
// read (GQA reuse): all G = nq/nkv heads of the kv head, or a group of 4 when
// the batch is too small to fill the GPU otherwise (attn_core.cuh).  Scores are fp32 (q.k of bf16 inputs,
// then * scale, as in the reference), softmax is fp32 with a split-local max;
// the last CTA of each (b, kvh) merges the splits (flash-decoding combine).
// Probabilities stay fp32 up to the P.V sum (the reference rounds them to bf16
// first); the output is rounded to bf16 once.
#include <math.h>

#include "attn_core.cuh"
#include "common.cuh"
#include "launch.cuh"

namespace jsx {

__global__ void __launch_bounds__(kAttnThreads) k_attn_decode(AttnArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  pdl_wait();
  attn_item_any<kAttnThreads, false, false>(a, blockIdx.x, blockIdx.y, smem_raw);
}

// Split merge as its own launch, one CTA per (item group, head), when a group's
// records do not fit the items' shared memory (large batches: 16-head groups of
// many sequences).  The last-arriving split would otherwise merge them from L2
// with one dependent round trip per few splits and output vectors, ~20 us at
// 32 sequences; here each thread owns one output dimension and has all its
// splits' loads in flight.  Same arithmetic and order as attn_finish's L2 form:
// M = max over splits, L = sum of l_t exp(m_t - M) in split order,
// out = sum_t fma(acc_t, exp(m_t - M) / L) in split order.
__global__ void __launch_bounds__(kAttnThreads) k_attn_merge(AttnArgs a) {
  pdl_wait();
  const int vb = blockIdx.y, h = blockIdx.x;  // group, head inside the group
  const int gi = a.gi, hd = a.hd, stride = split_stride(gi, hd);
  const int b = vb / (a.nkv * a.hg);
  const int kvh = (vb / a.hg) % a.nkv, j = vb % a.hg;
  const int head = kvh * (a.nq / a.nkv) + j * gi + h;
  int cur = a.pos[b];
  if (cur > a.max_seq - 1) cur = a.max_seq - 1;
  if (cur < 0) cur = 0;
  const int used = (cur + kChunk) / kChunk;
  const float* pb = a.part + (size_t)vb * a.splits * stride;
  __shared__ float w[1024];
  if (threadIdx.x == 0) {
    float M = -INFINITY;
    for (int t = 0; t < used; ++t) M = fmaxf(M, __ldcg(pb + (size_t)t * stride + gi * hd + h));
    float L = 0.f;
    for (int t = 0; t < used; ++t) {
      const float e = expf(__ldcg(pb + (size_t)t * stride + gi * hd + h) - M);
      w[t] = e;
      L = fmaf(__ldcg(pb + (size_t)t * stride + gi * hd + gi + h), e, L);
    }
    for (int t = 0; t < used; ++t) w[t] = expf(__ldcg(pb + (size_t)t * stride + gi * hd + h) - M) / L;
  }
  __syncthreads();
  bf16* ob = a.out + ((size_t)b * a.nq + head) * hd;
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float o = 0.f;
    for (int t0 = 0; t0 < used; t0 += 16) {
      float v[16];
#pragma unroll
      for (int u = 0; u < 16; ++u)
        v[u] = t0 + u < used ? __ldcg(pb + (size_t)(t0 + u) * stride + (size_t)h * hd + d) : 0.f;
#pragma unroll
      for (int u = 0; u < 16; ++u)
        if (t0 + u < used) o = fmaf(v[u], w[t0 + u], o);
    }
    ob[d] = __float2bfloat16_rn(o);
  }
  pdl_launch_dependents();
}

}  // namespace jsx

using namespace jsx;

extern "C" int jsx_attn_decode_workspace_size(int B, int nq, int nkv, int head_dim, int max_seq,
                                              size_t* bytes) {
  JSX_REQUIRE(bytes && B >= 1 && nq >= 1 && nkv >= 1 && nq % nkv == 0 && head_dim >= 2 &&
                  max_seq >= 1,
              "bad attention shape");
  *bytes = attn_layout(B, nq, nkv, head_dim, max_seq).bytes;
  return JSX_OK;
}

namespace jsx {

// Argument checks of jsx_attn_decode other than the workspace (shared with
// jsx_attn_decode_noalloc, which must reject a call before it touches its
// static scratch).
int attn_decode_check(const void* q, const void* k_cache, const void* v_cache, const void* out,
                      const int32_t* positions, int B, int nq, int nkv, int head_dim, int max_seq) {
  JSX_REQUIRE(q && k_cache && v_cache && out && positions, "null pointer argument");
  JSX_REQUIRE(B >= 1 && nq >= 1 && nkv >= 1 && nq % nkv == 0, "bad heads nq=%d nkv=%d", nq, nkv);
  JSX_REQUIRE(head_dim >= 8 && head_dim % 8 == 0 && head_dim <= 512, "head_dim=%d must be a multiple of 8",
              head_dim);
  JSX_REQUIRE(max_seq >= 1, "max_seq=%d", max_seq);
  JSX_REQUIRE(aligned16(k_cache) && aligned16(v_cache) && aligned16(out),
              "caches and out must be 16-byte aligned");
  const AttnLayout lay = attn_layout(B, nq, nkv, head_dim, max_seq);
  JSX_REQUIRE(attn_smem(lay.gi, head_dim, lay.splits) <= 200 * 1024, "attention tile too large (G=%d hd=%d)",
              nq / nkv, head_dim);
  return JSX_OK;
}

}  // namespace jsx

extern "C" int jsx_attn_decode(const void* q, const void* k_cache, const void* v_cache, void* out,
                               const int32_t* positions, int B, int nq, int nkv, int head_dim,
                               int max_seq, float scale, void* workspace, size_t workspace_bytes,
                               void* stream) {
  const int st = attn_decode_check(q, k_cache, v_cache, out, positions, B, nq, nkv, head_dim, max_seq);
  if (st != JSX_OK) return st;
  size_t need = 0;
  jsx_attn_decode_workspace_size(B, nq, nkv, head_dim, max_seq, &need);
  JSX_REQUIRE(workspace && workspace_bytes >= need && aligned16(workspace),
              "workspace of %zu bytes (16-byte aligned) required, got %zu", need, workspace_bytes);
  const AttnLayout lay = attn_layout(B, nq, nkv, head_dim, max_seq);
  const int splits = lay.splits;
  const size_t smem = attn_smem(lay.gi, head_dim, splits);
  AttnArgs a;
  a.q = (const bf16*)q; a.kc = (const bf16*)k_cache; a.vc = (const bf16*)v_cache;
  a.out = (bf16*)out; a.pos = positions; a.B = B; a.nq = nq; a.nkv = nkv; a.hd = head_dim;
  a.max_seq = max_seq; a.splits = splits; a.scale = scale;
  a.gi = lay.gi; a.hg = lay.hg;
  a.trace = nullptr;
  a.cnt = (uint32_t*)((char*)workspace + 256);
  a.part = (float*)((char*)workspace + lay.counter_bytes);
  // the last split merges its group from shared memory when the records fit there
  // (attn_finish); otherwise a merge launch does it (k_attn_merge)
  const size_t merge_need = (size_t)lay.splits * (lay.stride + lay.gi) * 4;
  const size_t scratch_off = attn_use_mma(lay.gi, head_dim) ? (size_t)kMmaHeads * kRowPad * 2
                                                             : (size_t)lay.gi * head_dim * 4 + (size_t)lay.gi * kChunk * 4;
  a.no_merge = (scratch_off + merge_need > smem && lay.splits <= 1024) ? 1 : 0;
  auto kern = k_attn_decode;
  JSX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  JSX_CUDA(launch_kernel(kern, dim3(a.splits, B * nkv * lay.hg), dim3(kAttnThreads), smem,
                         (cudaStream_t)stream, a));
  if (a.no_merge)
    JSX_CUDA(launch_kernel(k_attn_merge, dim3(lay.gi, B * nkv * lay.hg), dim3(kAttnThreads), 0, (cudaStream_t)stream,
                           a));
  return JSX_OK;
}
