// MLA decode in the absorbed-weight form over a latent cache (GLM-4.7-Flash,
// layers/mla_attention.py:101-193 computes the expanded form; this is the
// latent-cache decode the reference's own analysis names as its fix,
// README.md:67).
//
// The cache keeps, per token, the RMS-normalised kv latent c (kv_lora values)
// and the rotated shared rope key kr (rope values): 576 bf16 per token for
// GLM-4.7-Flash instead of nh * (nope + rope + v) = 20 * 512 expanded.  With
// W_k[h], W_v[h] the key and value columns of kv_b for head h:
//   q_abs[h] = bf16(W_k[h] q_nope[h])                          (jsx_mla_absorb)
//   s[h][t]  = bf16(bf16(q_abs[h] . c_t + q_rope[h] . kr_t) * scale)
//   ctx[h]   = bf16(softmax_t(s[h]) . c)                       (jsx_mla_decode)
//   out[h]   = bf16(W_v[h] ctx[h])                             (jsx_mla_absorb)
// Every head reads the same cache rows: one multi-query attention with a
// 576-wide key whose first kv_lora columns are also the value.
//
// jsx_mla_decode: one CTA per (sequence, 64-row split) stages the split's
// latent rows in shared memory once for all heads; S = Q K^T and O = P V run
// on mma.sync m16n8k16 with the heads as M (padded to 16 or 32); each split
// writes (acc, m, l); k_mla_merge combines the splits per (sequence, head)
// (flash-decoding combine) in a second, PDL-chained launch.
#include <math.h>

#include "attn_core.cuh"
#include "common.cuh"
#include "launch.cuh"

namespace jsx {

constexpr int kMlaRows = 64;       // cache rows per split
constexpr int kMlaThreads = 256;
constexpr int kMlaMaxDim = 576;    // kv_lora + rope handled by the decode kernel (multiples of 16)
constexpr int kMlaMaxHeadTiles = 2;

// ---------------------------------------------------------------------------
// latent cache write + RoPE of the query's rope slice
// ---------------------------------------------------------------------------
struct MlaLatentArgs {
  const bf16* q_in;    // [M][nh][nope + rope]
  const bf16* c;       // [M][kv_lora] normalised latent
  const bf16* k_rope;  // [M][rope] (kv_a_proj_with_mqa's rope columns, before RoPE)
  const float* inv_freq;
  const int32_t* pos;
  bf16* q_rope;        // [M][nh][rope] rotated
  bf16* latent;        // [B][max_seq][kv_lora + rope]
  int M, tps, nh, nope, rope, kv_lora, max_seq;
};

// layers/rotary.py:56-58, :88-91 (rotary_dim = rope): fp32 angle, bf16 cos/sin,
// neox half split, every product and sum rounded to bf16.
__device__ __forceinline__ void mla_rope_pair(float x1, float x2, float ang, float& o1, float& o2) {
  float s, c;
  sincosf(ang, &s, &c);
  c = rbf(c);
  s = rbf(s);
  o1 = rbf(rbf(x1 * c) - rbf(x2 * s));
  o2 = rbf(rbf(x2 * c) + rbf(x1 * s));
}

__global__ void __launch_bounds__(256) k_mla_latent_cache(MlaLatentArgs a) {
  pdl_wait();
  const int m = blockIdx.x;
  const int p = a.pos[m];
  const int half = a.rope >> 1;
  const int slot = p < 0 ? 0 : (p >= a.max_seq ? a.max_seq - 1 : p);  // dynamic_update_slice clamp
  const int b = m / a.tps;
  const int D = a.kv_lora + a.rope;
  bf16* row = a.latent + ((size_t)b * a.max_seq + slot) * D;
  for (int i = threadIdx.x; i < a.kv_lora; i += blockDim.x) row[i] = a.c[(size_t)m * a.kv_lora + i];
  for (int j = threadIdx.x; j < half; j += blockDim.x) {
    const float ang = (float)p * a.inv_freq[j];
    const bf16* kr = a.k_rope + (size_t)m * a.rope;
    float o1, o2;
    mla_rope_pair(__bfloat162float(kr[j]), __bfloat162float(kr[j + half]), ang, o1, o2);
    row[a.kv_lora + j] = __float2bfloat16_rn(o1);
    row[a.kv_lora + j + half] = __float2bfloat16_rn(o2);
  }
  for (int i = threadIdx.x; i < a.nh * half; i += blockDim.x) {
    const int h = i / half, j = i - h * half;
    const float ang = (float)p * a.inv_freq[j];
    const bf16* q = a.q_in + ((size_t)m * a.nh + h) * (a.nope + a.rope) + a.nope;
    float o1, o2;
    mla_rope_pair(__bfloat162float(q[j]), __bfloat162float(q[j + half]), ang, o1, o2);
    bf16* qo = a.q_rope + ((size_t)m * a.nh + h) * a.rope;
    qo[j] = __float2bfloat16_rn(o1);
    qo[j + half] = __float2bfloat16_rn(o2);
  }
}

// ---------------------------------------------------------------------------
// per-head absorption GEMV: out[m][h][r] = bf16(sum_k w[h][r][k] x[m][h][k])
// ---------------------------------------------------------------------------
struct MlaAbsorbArgs {
  const bf16* x;   // token m, head h at x + m * x_tok + h * x_head (K contiguous values)
  const bf16* w;   // [nh][R][K]
  bf16* out;       // [M][nh][R]
  int M, nh, R, K;
  int x_tok, x_head;
};

constexpr int kAbsorbRowsPerCta = 64;
constexpr int kAbsorbMaxTokens = 32;
constexpr int kAbsorbMaxK = 512;

// Sum of v[0..7] over the 32 lanes of a warp, 9 shuffles: afterwards lanes
// with (lane & 3) == 0 hold the total of token ((lane >> 4) & 1) * 4 +
// ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1) in v[0].
__device__ __forceinline__ void warp_sum8(float (&v)[8], int lane) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const bool up = lane & 16;
    const float send = up ? v[j] : v[j + 4];
    const float keep = up ? v[j + 4] : v[j];
    v[j] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const bool up = lane & 8;
    const float send = up ? v[j] : v[j + 2];
    const float keep = up ? v[j + 2] : v[j];
    v[j] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  {
    const bool up = lane & 4;
    const float send = up ? v[0] : v[1];
    const float keep = up ? v[1] : v[0];
    v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  v[0] += __shfl_xor_sync(0xffffffffu, v[0], 2);
  v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
}

__global__ void __launch_bounds__(256) k_mla_absorb(MlaAbsorbArgs a) {
  __shared__ __align__(16) bf16 xs[kAbsorbMaxTokens * kAbsorbMaxK];
  const int h = blockIdx.y;
  const int nvec = a.K >> 3;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // this CTA's weight rows do not depend on the previous kernel: the first
  // row's vectors are loaded before waiting on it
  const int r_first = blockIdx.x * kAbsorbRowsPerCta + warp;
  const uint4* wh = reinterpret_cast<const uint4*>(a.w) + (size_t)h * a.R * nvec;
  uint4 wv0 = make_uint4(0, 0, 0, 0), wv1 = make_uint4(0, 0, 0, 0);
  if (r_first < a.R) {
    if (lane < nvec) wv0 = ld_stream(wh + (size_t)r_first * nvec + lane);
    if (lane + 32 < nvec) wv1 = ld_stream(wh + (size_t)r_first * nvec + lane + 32);
  }
  pdl_wait();
  for (int i = threadIdx.x; i < a.M * nvec; i += blockDim.x) {
    const int m = i / nvec, v = i - m * nvec;
    reinterpret_cast<uint4*>(xs)[i] =
        reinterpret_cast<const uint4*>(a.x + (size_t)m * a.x_tok + (size_t)h * a.x_head)[v];
  }
  __syncthreads();
  const int r_end = min(a.R, (int)(blockIdx.x + 1) * kAbsorbRowsPerCta);
  for (int r = r_first; r < r_end; r += 8) {
    if (r != r_first) {
      wv0 = lane < nvec ? ld_stream(wh + (size_t)r * nvec + lane) : make_uint4(0, 0, 0, 0);
      wv1 = lane + 32 < nvec ? ld_stream(wh + (size_t)r * nvec + lane + 32) : make_uint4(0, 0, 0, 0);
    }
    float w0[8], w1[8];
    unpack8(wv0, w0);
    unpack8(wv1, w1);
    for (int m0 = 0; m0 < a.M; m0 += 8) {
      float acc[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        acc[t] = 0.f;
        const int m = m0 + t;
        if (m < a.M) {
          if (lane < nvec) {
            float xf[8];
            unpack8(reinterpret_cast<const uint4*>(xs)[m * nvec + lane], xf);
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[t] = fmaf(w0[j], xf[j], acc[t]);
          }
          if (lane + 32 < nvec) {
            float xf[8];
            unpack8(reinterpret_cast<const uint4*>(xs)[m * nvec + lane + 32], xf);
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[t] = fmaf(w1[j], xf[j], acc[t]);
          }
        }
      }
      warp_sum8(acc, lane);
      const int t = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
      if ((lane & 3) == 0 && m0 + t < a.M)
        a.out[((size_t)(m0 + t) * a.nh + h) * a.R + r] = __float2bfloat16_rn(acc[0]);
    }
  }
  pdl_launch_dependents();
}

// ---------------------------------------------------------------------------
// multi-query attention over the latent cache, split over the context
// ---------------------------------------------------------------------------
struct MlaDecodeArgs {
  const bf16* q_abs;   // [B][nh][kv_lora]
  const bf16* q_rope;  // [B][nh][rope]
  const bf16* latent;  // [B][max_seq][kv_lora + rope]
  bf16* ctx;           // [B][nh][kv_lora]
  const int32_t* pos;
  float* part;         // [B][splits][rec]: acc [nh][kv_lora], then m [nh], l [nh] (padded to 4)
  int B, nh, kv_lora, rope, max_seq, splits, rec;
  float scale;
};

__host__ __device__ __forceinline__ int mla_rec_floats(int nh, int kv_lora) {
  return nh * kv_lora + ((2 * nh + 3) & ~3);
}

// shared layout (bf16 rows padded by 8 elements: 16-byte aligned, conflict-free ldmatrix)
__host__ __device__ __forceinline__ int mla_row_pad(int D) { return D + 8; }
__host__ __device__ __forceinline__ size_t mla_decode_smem(int head_tiles, int D) {
  const int rp = mla_row_pad(D);
  return (size_t)head_tiles * 16 * rp * 2 + (size_t)kMlaRows * rp * 2 +          // q, latent rows
         (size_t)head_tiles * 16 * kMlaRows * 4 + (size_t)head_tiles * 16 * (kMlaRows + 8) * 2;  // S, P
}

template <int HT>
__global__ void __launch_bounds__(kMlaThreads) k_mla_decode(MlaDecodeArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  constexpr int NW = kMlaThreads / 32;
  constexpr int PP = kMlaRows + 8;
  const int D = a.kv_lora + a.rope, rp = mla_row_pad(D);
  bf16* qs = reinterpret_cast<bf16*>(smem_raw);      // [HT*16][rp]: q_abs | q_rope, rows >= nh zero
  bf16* ks = qs + HT * 16 * rp;                      // [64][rp]: latent rows (value = first kv_lora)
  float* ss = reinterpret_cast<float*>(ks + kMlaRows * rp);  // [HT*16][64] scores
  bf16* ps = reinterpret_cast<bf16*>(ss + HT * 16 * kMlaRows);  // [HT*16][PP] probabilities

  const int s = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int p0 = s * kMlaRows;
  const int dv = D >> 3;  // 16-byte vectors per row
  // cache rows written by earlier steps do not depend on the previous kernel:
  // stage the rows below the position before waiting on it (the position is
  // written by the host or an earlier graph node, not by the previous kernel)
  int cur = a.pos[b];
  if (cur > a.max_seq - 1) cur = a.max_seq - 1;
  if (cur < 0) cur = 0;
  int n = cur + 1 - p0;  // rows of this split inside [0, cur]
  if (n > kMlaRows) n = kMlaRows;
  const bf16* lb = a.latent + ((size_t)b * a.max_seq + p0) * D;
  for (int i = tid; i < kMlaRows * dv; i += kMlaThreads) {
    const int r = i / dv, c = i - r * dv;
    if (r == n - 1 && p0 + r == cur) continue;  // this step's row: after the wait
    const bool live = r < n;
    cp_async16(ks + r * rp + c * 8, lb + (size_t)(live ? r : 0) * D + c * 8, live ? 16u : 0u);
  }
  pdl_wait();
  if (n > 0 && n - 1 + p0 == cur) {
    for (int c = tid; c < dv; c += kMlaThreads) cp_async16(ks + (n - 1) * rp + c * 8, lb + (size_t)(n - 1) * D + c * 8, 16u);
  }
  const int qv_abs = a.kv_lora >> 3;
  for (int i = tid; i < HT * 16 * dv; i += kMlaThreads) {
    const int h = i / dv, c = i - h * dv;
    const bool live = h < a.nh;
    const bf16* src = c < qv_abs ? a.q_abs + ((size_t)b * a.nh + (live ? h : 0)) * a.kv_lora + c * 8
                                 : a.q_rope + ((size_t)b * a.nh + (live ? h : 0)) * a.rope + (c - qv_abs) * 8;
    cp_async16(qs + h * rp + c * 8, src, live ? 16u : 0u);
  }
  cp_async_wait_all();
  __syncthreads();

  float* part = a.part + ((size_t)b * a.splits + s) * a.rec;
  if (n > 0) {
    const int g = lane >> 2, t4 = lane & 3;
    // S = Q K^T: warp w owns score rows [8w, 8w + 8) for every head tile
    {
      float sc[HT][4];
#pragma unroll
      for (int ht = 0; ht < HT; ++ht) sc[ht][0] = sc[ht][1] = sc[ht][2] = sc[ht][3] = 0.f;
      for (int kk = 0; kk < D / 16; ++kk) {
        uint32_t b0, b1;
        ldsm_x2(smem_addr(ks + (8 * warp + (lane & 7)) * rp + 16 * kk + ((lane >> 3) & 1) * 8), b0, b1);
#pragma unroll
        for (int ht = 0; ht < HT; ++ht) {
          uint32_t a0, a1, a2, a3;
          ldsm_x4(smem_addr(qs + (16 * ht + (lane & 15)) * rp + 16 * kk + (lane >> 4) * 8), a0, a1, a2, a3);
          mma_bf16_16816(sc[ht], a0, a1, a2, a3, b0, b1);
        }
      }
      // the reference rounds q.k to bf16, then the scaled score to bf16 (mla_attention.py:176-184)
      const int r = 8 * warp + 2 * t4;
#pragma unroll
      for (int ht = 0; ht < HT; ++ht) {
        const int h0 = 16 * ht + g;
        ss[h0 * kMlaRows + r] = r < n ? rbf(rbf(sc[ht][0]) * a.scale) : -INFINITY;
        ss[h0 * kMlaRows + r + 1] = r + 1 < n ? rbf(rbf(sc[ht][1]) * a.scale) : -INFINITY;
        ss[(h0 + 8) * kMlaRows + r] = r < n ? rbf(rbf(sc[ht][2]) * a.scale) : -INFINITY;
        ss[(h0 + 8) * kMlaRows + r + 1] = r + 1 < n ? rbf(rbf(sc[ht][3]) * a.scale) : -INFINITY;
      }
    }
    __syncthreads();
    // split-local softmax pieces per head: m, e = exp(s - m) (bf16 for the MMA), l (fp32)
    for (int h = warp; h < HT * 16; h += NW) {
      if (h >= a.nh) {
        ps[h * PP + lane] = __float2bfloat16_rn(0.f);
        ps[h * PP + lane + 32] = __float2bfloat16_rn(0.f);
        continue;
      }
      const float v0 = ss[h * kMlaRows + lane], v1 = ss[h * kMlaRows + lane + 32];
      const float m = warp_max(fmaxf(v0, v1));
      const float e0 = lane < n ? expf(v0 - m) : 0.f;
      const float e1 = lane + 32 < n ? expf(v1 - m) : 0.f;
      ps[h * PP + lane] = __float2bfloat16_rn(e0);
      ps[h * PP + lane + 32] = __float2bfloat16_rn(e1);
      const float l = warp_sum(e0 + e1);
      if (lane == 0) {
        part[a.nh * a.kv_lora + h] = m;
        part[a.nh * a.kv_lora + a.nh + h] = l;
      }
    }
    __syncthreads();
    // O = P V over the value columns [0, kv_lora): warp w owns dims [dw w, dw w + dw)
    const int dw = a.kv_lora / NW;  // 64 for kv_lora 512
    for (int d0 = dw * warp; d0 < dw * (warp + 1); d0 += 32) {
      float o[HT][4][4];
#pragma unroll
      for (int ht = 0; ht < HT; ++ht)
#pragma unroll
        for (int jn = 0; jn < 4; ++jn) o[ht][jn][0] = o[ht][jn][1] = o[ht][jn][2] = o[ht][jn][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < kMlaRows / 16; ++kk) {
        uint32_t bb[4][2];
#pragma unroll
        for (int jn = 0; jn < 4; ++jn)
          ldsm_x2_t(smem_addr(ks + (16 * kk + (lane & 7) + ((lane >> 3) & 1) * 8) * rp + d0 + 8 * jn), bb[jn][0],
                    bb[jn][1]);
#pragma unroll
        for (int ht = 0; ht < HT; ++ht) {
          uint32_t a0, a1, a2, a3;
          ldsm_x4(smem_addr(ps + (16 * ht + (lane & 15)) * PP + 16 * kk + (lane >> 4) * 8), a0, a1, a2, a3);
#pragma unroll
          for (int jn = 0; jn < 4; ++jn) mma_bf16_16816(o[ht][jn], a0, a1, a2, a3, bb[jn][0], bb[jn][1]);
        }
      }
#pragma unroll
      for (int ht = 0; ht < HT; ++ht) {
        const int h0 = 16 * ht + g;
#pragma unroll
        for (int jn = 0; jn < 4; ++jn) {
          const int d = d0 + 8 * jn + 2 * t4;
          if (h0 < a.nh)
            *reinterpret_cast<float2*>(part + (size_t)h0 * a.kv_lora + d) = make_float2(o[ht][jn][0], o[ht][jn][1]);
          if (h0 + 8 < a.nh)
            *reinterpret_cast<float2*>(part + (size_t)(h0 + 8) * a.kv_lora + d) =
                make_float2(o[ht][jn][2], o[ht][jn][3]);
        }
      }
    }
  }
  pdl_launch_dependents();
}

// Combine of the splits of one (sequence, head): w_s = exp(m_s - M) / L,
// ctx = bf16(sum_s w_s acc_s).  Splits past the position hold nothing and are
// not read.
__global__ void __launch_bounds__(128) k_mla_merge(MlaDecodeArgs a) {
  __shared__ float w[1024];
  __shared__ float ML[2];
  const int h = blockIdx.x, b = blockIdx.y;
  pdl_wait();
  int cur = a.pos[b];
  if (cur > a.max_seq - 1) cur = a.max_seq - 1;
  if (cur < 0) cur = 0;
  const int used = cur / kMlaRows + 1;
  const float* pb = a.part + (size_t)b * a.splits * a.rec;
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    float M = -INFINITY;
    for (int t = lane; t < used; t += 32) M = fmaxf(M, __ldcg(pb + (size_t)t * a.rec + a.nh * a.kv_lora + h));
    M = warp_max(M);
    float L = 0.f;
    for (int t = lane; t < used; t += 32) {
      const float e = expf(__ldcg(pb + (size_t)t * a.rec + a.nh * a.kv_lora + h) - M);
      w[t] = e;
      L = fmaf(__ldcg(pb + (size_t)t * a.rec + a.nh * a.kv_lora + a.nh + h), e, L);
    }
    L = warp_sum(L);
    if (lane == 0) ML[1] = L;
  }
  __syncthreads();
  const float L = ML[1];
  bf16* ob = a.ctx + ((size_t)b * a.nh + h) * a.kv_lora;
  for (int d = threadIdx.x * 4; d < a.kv_lora; d += blockDim.x * 4) {
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int t = 0; t < used; ++t) {
      const float wt = w[t] / L;
      const float4 v = __ldcg(reinterpret_cast<const float4*>(pb + (size_t)t * a.rec + (size_t)h * a.kv_lora + d));
      o.x = fmaf(v.x, wt, o.x);
      o.y = fmaf(v.y, wt, o.y);
      o.z = fmaf(v.z, wt, o.z);
      o.w = fmaf(v.w, wt, o.w);
    }
    uint2 packed;
    packed.x = pack2(o.x, o.y);
    packed.y = pack2(o.z, o.w);
    *reinterpret_cast<uint2*>(ob + d) = packed;
  }
  pdl_launch_dependents();
}

}  // namespace jsx

using namespace jsx;

extern "C" int jsx_mla_latent_cache(const void* q_in, const void* c, const void* k_rope, const float* inv_freq,
                                    const int32_t* positions, void* q_rope, void* latent_cache, int M,
                                    int tokens_per_seq, int nh, int nope, int rope, int kv_lora, int max_seq,
                                    void* stream) {
  JSX_REQUIRE(q_in && c && k_rope && inv_freq && positions && q_rope && latent_cache, "null pointer argument");
  JSX_REQUIRE(M >= 1 && tokens_per_seq >= 1 && M % tokens_per_seq == 0, "M=%d tokens_per_seq=%d", M,
              tokens_per_seq);
  JSX_REQUIRE(nh >= 1 && nope >= 0 && rope >= 2 && rope % 2 == 0 && kv_lora >= 1 && max_seq >= 1,
              "bad MLA shape nh=%d nope=%d rope=%d kv_lora=%d", nh, nope, rope, kv_lora);
  MlaLatentArgs a;
  a.q_in = (const bf16*)q_in; a.c = (const bf16*)c; a.k_rope = (const bf16*)k_rope; a.inv_freq = inv_freq;
  a.pos = positions; a.q_rope = (bf16*)q_rope; a.latent = (bf16*)latent_cache;
  a.M = M; a.tps = tokens_per_seq; a.nh = nh; a.nope = nope; a.rope = rope; a.kv_lora = kv_lora;
  a.max_seq = max_seq;
  JSX_CUDA(launch_kernel(k_mla_latent_cache, dim3(M), dim3(256), 0, (cudaStream_t)stream, a));
  return JSX_OK;
}

extern "C" int jsx_mla_absorb(const void* x, int x_token_stride, int x_head_stride, const void* w, void* out,
                              int M, int nh, int R, int K, void* stream) {
  JSX_REQUIRE(x && w && out, "null pointer argument");
  JSX_REQUIRE(M >= 1 && M <= kAbsorbMaxTokens, "M=%d outside 1..%d", M, kAbsorbMaxTokens);
  JSX_REQUIRE(nh >= 1 && nh <= 65535 && R >= 1, "nh=%d R=%d", nh, R);
  JSX_REQUIRE(K >= 8 && K % 8 == 0 && K <= kAbsorbMaxK, "K=%d must be a multiple of 8 up to %d", K, kAbsorbMaxK);
  JSX_REQUIRE(x_token_stride % 8 == 0 && x_head_stride % 8 == 0 && aligned16(x) && aligned16(w),
              "x strides must be multiples of 8 elements and x, w 16-byte aligned");
  MlaAbsorbArgs a;
  a.x = (const bf16*)x; a.w = (const bf16*)w; a.out = (bf16*)out;
  a.M = M; a.nh = nh; a.R = R; a.K = K; a.x_tok = x_token_stride; a.x_head = x_head_stride;
  const dim3 grid((R + kAbsorbRowsPerCta - 1) / kAbsorbRowsPerCta, nh);
  JSX_CUDA(launch_kernel(k_mla_absorb, grid, dim3(256), 0, (cudaStream_t)stream, a));
  return JSX_OK;
}

extern "C" int jsx_mla_decode_workspace_size(int B, int nh, int kv_lora, int max_seq, size_t* bytes) {
  JSX_REQUIRE(bytes && B >= 1 && nh >= 1 && kv_lora >= 1 && max_seq >= 1, "bad MLA decode shape");
  const int splits = (max_seq + kMlaRows - 1) / kMlaRows;
  *bytes = (size_t)B * splits * mla_rec_floats(nh, kv_lora) * sizeof(float);
  return JSX_OK;
}

extern "C" int jsx_mla_decode(const void* q_abs, const void* q_rope, const void* latent_cache, void* ctx,
                              const int32_t* positions, int B, int nh, int kv_lora, int rope, int max_seq,
                              float scale, void* workspace, size_t workspace_bytes, void* stream) {
  JSX_REQUIRE(q_abs && q_rope && latent_cache && ctx && positions && workspace, "null pointer argument");
  JSX_REQUIRE(B >= 1 && B <= 65535 && max_seq >= 1, "B=%d max_seq=%d", B, max_seq);
  JSX_REQUIRE(nh >= 1 && nh <= 16 * kMlaMaxHeadTiles, "nh=%d outside 1..%d", nh, 16 * kMlaMaxHeadTiles);
  JSX_REQUIRE(kv_lora % 256 == 0 && kv_lora >= 256 && rope % 16 == 0 && rope >= 16 && kv_lora + rope <= kMlaMaxDim,
              "kv_lora=%d (multiple of 256) + rope=%d (multiple of 16) must be at most %d", kv_lora, rope,
              kMlaMaxDim);
  JSX_REQUIRE((max_seq + kMlaRows - 1) / kMlaRows <= 1024, "max_seq=%d exceeds %d", max_seq, 1024 * kMlaRows);
  JSX_REQUIRE(aligned16(q_abs) && aligned16(q_rope) && aligned16(latent_cache) && aligned16(ctx) &&
                  aligned16(workspace),
              "tensors must be 16-byte aligned");
  size_t need = 0;
  jsx_mla_decode_workspace_size(B, nh, kv_lora, max_seq, &need);
  JSX_REQUIRE(workspace_bytes >= need, "workspace of %zu bytes required, got %zu", need, workspace_bytes);
  MlaDecodeArgs a;
  a.q_abs = (const bf16*)q_abs; a.q_rope = (const bf16*)q_rope; a.latent = (const bf16*)latent_cache;
  a.ctx = (bf16*)ctx; a.pos = positions; a.part = (float*)workspace;
  a.B = B; a.nh = nh; a.kv_lora = kv_lora; a.rope = rope; a.max_seq = max_seq;
  a.splits = (max_seq + kMlaRows - 1) / kMlaRows;
  a.rec = mla_rec_floats(nh, kv_lora);
  a.scale = scale;
  const int HT = nh <= 16 ? 1 : 2;
  const size_t smem = mla_decode_smem(HT, kv_lora + rope);
  const dim3 grid(a.splits, B);
  if (HT == 1) {
    JSX_CUDA(cudaFuncSetAttribute(k_mla_decode<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    JSX_CUDA(launch_kernel(k_mla_decode<1>, grid, dim3(kMlaThreads), smem, (cudaStream_t)stream, a));
  } else {
    JSX_CUDA(cudaFuncSetAttribute(k_mla_decode<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    JSX_CUDA(launch_kernel(k_mla_decode<2>, grid, dim3(kMlaThreads), smem, (cudaStream_t)stream, a));
  }
  JSX_CUDA(launch_kernel(k_mla_merge, dim3(nh, B), dim3(128), 0, (cudaStream_t)stream, a));
  return JSX_OK;
}
