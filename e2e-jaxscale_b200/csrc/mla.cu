// MLA (GLM-4.7-Flash, layers/mla_attention.py:101-193): the step between the
// low-rank projections and the attention.  RoPE on the rope slice of every
// query head and on the shared rope key (broadcast to every head), the
// concatenation [nope | rope], and the expanded per-head cache write.
//
// The projections themselves are plain linear layers (jsx_linear; the latent
// RMSNorms run as the prologue of q_b / kv_b), the attention is jsx_attn_decode
// with one query head per kv head, o_proj is jsx_row_linear_allreduce.
#include <math.h>

#include "common.cuh"
#include "launch.cuh"

namespace jsx {

struct MlaArgs {
  const bf16* q_in;     // [M][nh][nope + rope]
  const bf16* kv_in;    // [M][nh][nope + vdim]
  const bf16* k_rope;   // [M][rope] shared rope key
  const float* inv_freq;
  const int32_t* pos;
  bf16* q_out;          // [M][nh][nope + rope]
  bf16* kc;             // [B][max_seq][nh][nope + rope]
  bf16* vc;             // [B][max_seq][nh][vdim]
  int M, tps, nh, nope, rope, vdim, max_seq;
};

// layers/rotary.py:56-58, :88-91 with rotary_dim = rope: fp32 angle, bf16 cos/sin,
// neox half split, every product and sum rounded to bf16.
__device__ __forceinline__ void rope_pair(float x1, float x2, float ang, float& o1, float& o2) {
  float s, c;
  sincosf(ang, &s, &c);
  c = rbf(c);
  s = rbf(s);
  o1 = rbf(rbf(x1 * c) - rbf(x2 * s));
  o2 = rbf(rbf(x2 * c) + rbf(x1 * s));
}

__global__ void __launch_bounds__(256) k_mla_rope_cache(MlaArgs a) {
  extern __shared__ float kr[];  // rotated shared key [rope]
  pdl_wait();
  pdl_launch_dependents();
  const int m = blockIdx.x;
  const int p = a.pos[m];
  const int half = a.rope >> 1;
  const int qd = a.nope + a.rope;
  for (int j = threadIdx.x; j < half; j += blockDim.x) {
    const bf16* k = a.k_rope + (size_t)m * a.rope;
    float o1, o2;
    rope_pair(ldbf(k + j), ldbf(k + j + half), (float)p * a.inv_freq[j], o1, o2);
    kr[j] = o1;
    kr[j + half] = o2;
  }
  __syncthreads();
  const int b = m / a.tps;
  // dynamic_update_slice clamps the start row into [0, max_seq - 1] (layers/mla_attention.py:160-166)
  const int slot = p < 0 ? 0 : (p >= a.max_seq ? a.max_seq - 1 : p);
  for (int h = 0; h < a.nh; ++h) {
    const bf16* qi = a.q_in + ((size_t)m * a.nh + h) * qd;
    bf16* qo = a.q_out + ((size_t)m * a.nh + h) * qd;
    const bf16* kvi = a.kv_in + ((size_t)m * a.nh + h) * (a.nope + a.vdim);
    bf16* kd = a.kc + (((size_t)b * a.max_seq + slot) * a.nh + h) * qd;
    bf16* vd = a.vc + (((size_t)b * a.max_seq + slot) * a.nh + h) * a.vdim;
    for (int d = threadIdx.x; d < a.nope; d += blockDim.x) {
      qo[d] = qi[d];
      kd[d] = kvi[d];
    }
    for (int j = threadIdx.x; j < half; j += blockDim.x) {
      float o1, o2;
      rope_pair(ldbf(qi + a.nope + j), ldbf(qi + a.nope + j + half), (float)p * a.inv_freq[j], o1, o2);
      qo[a.nope + j] = __float2bfloat16_rn(o1);
      qo[a.nope + j + half] = __float2bfloat16_rn(o2);
    }
    for (int j = threadIdx.x; j < a.rope; j += blockDim.x) kd[a.nope + j] = __float2bfloat16_rn(kr[j]);
    for (int d = threadIdx.x; d < a.vdim; d += blockDim.x) vd[d] = kvi[a.nope + d];
  }
}

}  // namespace jsx

using namespace jsx;

extern "C" int jsx_mla_rope_cache(const void* q_in, const void* kv_in, const void* k_rope, const float* inv_freq,
                                  const int32_t* positions, void* q_out, void* k_cache, void* v_cache, int M,
                                  int tokens_per_seq, int nh, int nope, int rope, int vdim, int max_seq,
                                  void* stream) {
  JSX_REQUIRE(q_in && kv_in && k_rope && inv_freq && positions && q_out && k_cache && v_cache,
              "null pointer argument");
  JSX_REQUIRE(M >= 1 && tokens_per_seq >= 1 && M % tokens_per_seq == 0, "M=%d tokens_per_seq=%d", M,
              tokens_per_seq);
  JSX_REQUIRE(nh >= 1 && nope >= 0 && rope >= 2 && rope % 2 == 0 && vdim >= 1 && max_seq >= 1,
              "nh=%d nope=%d rope=%d vdim=%d", nh, nope, rope, vdim);
  MlaArgs a;
  a.q_in = (const bf16*)q_in; a.kv_in = (const bf16*)kv_in; a.k_rope = (const bf16*)k_rope;
  a.inv_freq = inv_freq; a.pos = positions; a.q_out = (bf16*)q_out; a.kc = (bf16*)k_cache;
  a.vc = (bf16*)v_cache; a.M = M; a.tps = tokens_per_seq; a.nh = nh; a.nope = nope; a.rope = rope;
  a.vdim = vdim; a.max_seq = max_seq;
  JSX_CUDA(launch_kernel(k_mla_rope_cache, dim3(M), dim3(256), (size_t)rope * sizeof(float), (cudaStream_t)stream,
                         a));
  return JSX_OK;
}
