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
  a.no_merge = 0;
  a.dist_err = nullptr;  // splits of a group may not be co-resident: the last one merges
  a.cnt = (uint32_t*)((char*)workspace + 256);
  a.part = (float*)((char*)workspace + lay.counter_bytes);
  auto kern = k_attn_decode;
  JSX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  JSX_CUDA(launch_kernel(kern, dim3(a.splits, B * nkv * lay.hg), dim3(kAttnThreads), smem,
                         (cudaStream_t)stream, a));
  return JSX_OK;
}
