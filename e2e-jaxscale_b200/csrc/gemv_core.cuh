// Decode GEMV building blocks shared by the per-op kernels (gemv.cu) and the
// whole-step decode kernel (decode_step.cu): argument block, activation
// staging with the fused RMSNorm, register-streamed weight batches, and the
// value-level epilogues of the fused q/k/v (+RoPE, KV write) and gate/up
// (+SwiGLU) projections.
#pragma once

#include "comm.cuh"
#include "common.cuh"

namespace jsx {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kRows = 2;    // rows per warp group (the qkv / gate_up packings assume 2)
constexpr int kUnroll = 8;  // 16-byte vectors per lane per row in flight
constexpr int kMaxM = 8;
// dynamic shared memory a decode kernel may request (B200: 227 KB per CTA, less the static part)
constexpr size_t kMaxDynSmem = 225 * 1024;

enum Epi { EPI_LINEAR = 0, EPI_QKV = 1, EPI_SWIGLU = 2, EPI_ROWAR = 3, EPI_LMHEAD = 4 };

struct GemvArgs {
  const bf16* x;      // [M][K]
  const bf16* gamma;  // RMSNorm gain [K] or null
  float eps;
  const bf16* w;      // packed [N][K]
  int M, K, N;        // N = packed rows
  // EPI_LINEAR
  const bf16* bias;
  bf16* y;            // [M][N] (linear), q_out [M][nq*hd] (qkv), act [M][N/2] (swiglu)
  // EPI_QKV
  const float* inv_freq;
  const int32_t* pos;
  bf16* kc;
  bf16* vc;
  int nq, nkv, hd, rot, max_seq, tps;
  // EPI_ROWAR
  bf16* h;            // residual [M][N]
  const bf16* addend; // [M][N] added to this rank's partial before the all-reduce, or null
  // EPI_LMHEAD
  int vocab_offset;
  unsigned long long* keys;  // [M] workspace (zero on entry, left zero)
  uint32_t* done;            // workspace counter (zero on entry, left zero)
  int32_t* ids;              // [M]
};

// ---- activations -> shared memory (optionally RMS-normalised) --------------
// layers/normalization.py:31-37: y = bf16((x * rsqrt(mean(x^2) + eps)) * g), fp32 inside.
// Barrier over the threads that stage the activations: the whole CTA (v1
// kernel) or the 8 consumer warps of the streaming kernel (named barrier 1).
template <bool kNamed>
__device__ __forceinline__ void stage_sync() {
  if constexpr (kNamed) asm volatile("bar.sync 1, 256;" ::: "memory");
  else __syncthreads();
}

// kCoherent: read the activations with ld.global.cg (L2), for data another CTA
// of the same kernel wrote (the whole-step kernel); the per-op kernels read
// data of earlier kernels and may use L1.
__device__ __forceinline__ uint4 ld_act(const uint4* p, bool coherent) {
  return coherent ? __ldcg(p) : *p;
}

template <int M, bool kNamed = false, bool kCoherent = false>
__device__ __forceinline__ void stage_x(const GemvArgs& a, bf16* xs) {
  constexpr int NT = kThreads;  // 256 staging threads in both kernels
  const int nvec = a.K >> 3;
  const uint4* xv = reinterpret_cast<const uint4*>(a.x);
  uint4* sv = reinterpret_cast<uint4*>(xs);
  if (a.gamma == nullptr) {
    for (int i = threadIdx.x; i < M * nvec; i += NT) sv[i] = ld_act(xv + i, kCoherent);
    stage_sync<kNamed>();
    return;
  }
  __shared__ float red[M][kWarps];
  __shared__ float rstd[M];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint4* gv = reinterpret_cast<const uint4*>(a.gamma);
  if constexpr (M <= 2) {
    // one pass: every vector a thread needs (at most 2 per token, K <= 16 * NT)
    // is held in registers between the sum of squares and the scaling; same
    // summation order and arithmetic as the two-pass form below.  The weights
    // are loaded with the activations, so their latency (HBM, for a norm read
    // once per step) overlaps the reduction instead of following it.
    if (nvec <= 2 * NT) {
      uint4 xr[M][2], gr[2];
      float ss[M];
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const int v = threadIdx.x + jj * NT;
#pragma unroll
        for (int m = 0; m < M; ++m)
          xr[m][jj] = v < nvec ? ld_act(xv + m * nvec + v, kCoherent) : make_uint4(0, 0, 0, 0);
        gr[jj] = v < nvec ? gv[v] : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int m = 0; m < M; ++m) ss[m] = 0.f;
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        if (threadIdx.x + jj * NT < nvec) {
#pragma unroll
          for (int m = 0; m < M; ++m) {
            float f[8];
            unpack8(xr[m][jj], f);
#pragma unroll
            for (int j = 0; j < 8; ++j) ss[m] = fmaf(f[j], f[j], ss[m]);
          }
        }
      }
#pragma unroll
      for (int m = 0; m < M; ++m) {
        float s = warp_sum(ss[m]);
        if (lane == 0) red[m][warp] = s;
      }
      stage_sync<kNamed>();
      if (threadIdx.x < M) {
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) t += red[threadIdx.x][w];
        rstd[threadIdx.x] = 1.0f / sqrtf(t / (float)a.K + a.eps);
      }
      stage_sync<kNamed>();
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const int v = threadIdx.x + jj * NT;
        if (v < nvec) {
          float g[8];
          unpack8(gr[jj], g);
#pragma unroll
          for (int m = 0; m < M; ++m) {
            float f[8];
            unpack8(xr[m][jj], f);
            const float r = rstd[m];
            uint4 o;
            o.x = pack2((f[0] * r) * g[0], (f[1] * r) * g[1]);
            o.y = pack2((f[2] * r) * g[2], (f[3] * r) * g[3]);
            o.z = pack2((f[4] * r) * g[4], (f[5] * r) * g[5]);
            o.w = pack2((f[6] * r) * g[6], (f[7] * r) * g[7]);
            sv[m * nvec + v] = o;
          }
        }
      }
      stage_sync<kNamed>();
      return;
    }
  }
  float ss[M];
#pragma unroll
  for (int m = 0; m < M; ++m) ss[m] = 0.f;
  for (int v = threadIdx.x; v < nvec; v += NT) {
#pragma unroll
    for (int m = 0; m < M; ++m) {
      float f[8];
      unpack8(ld_act(xv + m * nvec + v, kCoherent), f);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss[m] = fmaf(f[j], f[j], ss[m]);
    }
  }
#pragma unroll
  for (int m = 0; m < M; ++m) {
    float s = warp_sum(ss[m]);
    if (lane == 0) red[m][warp] = s;
  }
  stage_sync<kNamed>();
  if (threadIdx.x < M) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) t += red[threadIdx.x][w];
    rstd[threadIdx.x] = 1.0f / sqrtf(t / (float)a.K + a.eps);
  }
  stage_sync<kNamed>();
  for (int i = threadIdx.x; i < M * nvec; i += NT) {
    const int m = i / nvec, v = i - m * nvec;
    float f[8], g[8];
    unpack8(ld_act(xv + i, kCoherent), f);
    unpack8(gv[v], g);
    const float r = rstd[m];
    uint4 o;
    o.x = pack2((f[0] * r) * g[0], (f[1] * r) * g[1]);
    o.y = pack2((f[2] * r) * g[2], (f[3] * r) * g[3]);
    o.z = pack2((f[4] * r) * g[4], (f[5] * r) * g[5]);
    o.w = pack2((f[6] * r) * g[6], (f[7] * r) * g[7]);
    sv[i] = o;
  }
  stage_sync<kNamed>();
}

// ---- weight batches -----------------------------------------------------------
struct Batch {
  uint4 w[kUnroll][kRows];
};

__device__ __forceinline__ void load_batch(Batch& b, const uint4* __restrict__ wv, int nvec,
                                           int base, int lane) {
#pragma unroll
  for (int u = 0; u < kUnroll; ++u) {
    const int v = base + u * 32 + lane;
#pragma unroll
    for (int r = 0; r < kRows; ++r)
      b.w[u][r] = (v < nvec) ? ld_stream(wv + (size_t)r * nvec + v) : make_uint4(0, 0, 0, 0);
  }
}

template <int M>
__device__ __forceinline__ void fma_batch(const Batch& b, const uint4* __restrict__ xv, int nvec,
                                          int base, int lane, float (&acc)[kRows][M]) {
#pragma unroll
  for (int u = 0; u < kUnroll; ++u) {
    const int v = base + u * 32 + lane;
    if (v < nvec) {
      float wf[kRows][8];
#pragma unroll
      for (int r = 0; r < kRows; ++r) unpack8(b.w[u][r], wf[r]);
#pragma unroll
      for (int m = 0; m < M; ++m) {
        float xf[8];
        unpack8(xv[m * nvec + v], xf);
#pragma unroll
        for (int r = 0; r < kRows; ++r)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[r][m] = fmaf(wf[r][j], xf[j], acc[r][m]);
      }
    }
  }
}

// Value (r, m) of a warp-reduced accumulator tile, selected without dynamic
// register indexing.
template <int M>
__device__ __forceinline__ float pick(const float (&acc)[kRows][M], int r, int m) {
  float v = 0.f;
#pragma unroll
  for (int rr = 0; rr < kRows; ++rr)
#pragma unroll
    for (int mm = 0; mm < M; ++mm)
      if (rr == r && mm == m) v = acc[rr][mm];
  return v;
}

// ---- epilogues ------------------------------------------------------------------
// qkv packing (jsx_pack_qkv): per head hd/2 groups; group j < rot/2 holds rows
// (j, j + rot/2) (a neox rotary pair), group j >= rot/2 holds the pass-through
// pair (rot + 2(j - rot/2), +1).  Heads: q (nq), then k (nkv), then v (nkv).
// Columns (in q | k | v order) of packed row pair g: its head and the two
// dimensions d0, d1; rotary pairs first.
struct QkvCols {
  int head, j, d0, d1;
  bool rotary;
};
__device__ __forceinline__ QkvCols qkv_cols(const GemvArgs& a, int g) {
  QkvCols q;
  const int gph = a.hd >> 1;
  q.head = g / gph;
  q.j = g - q.head * gph;
  const int rh = a.rot >> 1;
  if (q.j < rh) { q.d0 = q.j; q.d1 = q.j + rh; q.rotary = true; }
  else { q.d0 = a.rot + 2 * (q.j - rh); q.d1 = q.d0 + 1; q.rotary = false; }
  return q;
}

// The bias pair of packed row pair g (0 without a bias).
__device__ __forceinline__ void qkv_bias_pair(const GemvArgs& a, int g, float& b0, float& b1) {
  b0 = b1 = 0.f;
  if (a.bias) {
    const QkvCols q = qkv_cols(a, g);
    b0 = ldbf(a.bias + q.head * a.hd + q.d0);
    b1 = ldbf(a.bias + q.head * a.hd + q.d1);
  }
}

// Epilogue of row pair g for token m with its bias pair already loaded (b0, b1
// are read only when a.bias is set); positions and rotary frequencies from
// `pos` / `inv_freq` (a.pos / a.inv_freq, or copies of them in shared memory).
__device__ __forceinline__ void qkv_store_b(const GemvArgs& a, int g, int m, float acc0, float acc1, float b0,
                                            float b1, const int32_t* pos, const float* inv_freq) {
  const QkvCols q = qkv_cols(a, g);
  const int head = q.head, j = q.j, d0 = q.d0, d1 = q.d1;
  float x1 = rbf(acc0);
  float x2 = rbf(acc1);
  if (a.bias) {
    x1 = rbf(x1 + b0);
    x2 = rbf(x2 + b1);
  }
  const int p = pos[m];
  const bool is_v = head >= a.nq + a.nkv;
  if (q.rotary && !is_v) {
    // layers/rotary.py:56-58 (fp32 angle, bf16 cos/sin) and :88-91 (half split)
    float s, c;
    sincosf((float)p * inv_freq[j], &s, &c);
    c = rbf(c);
    s = rbf(s);
    const float o1 = rbf(rbf(x1 * c) - rbf(x2 * s));
    const float o2 = rbf(rbf(x2 * c) + rbf(x1 * s));
    x1 = o1;
    x2 = o2;
  }
  if (head < a.nq) {
    bf16* qo = a.y + (size_t)m * a.nq * a.hd + head * a.hd;
    qo[d0] = __float2bfloat16_rn(x1);
    qo[d1] = __float2bfloat16_rn(x2);
  } else {
    const int kvh = is_v ? head - a.nq - a.nkv : head - a.nq;
    const int b = m / a.tps;
    // dynamic_update_slice clamps the start row into [0, max_seq - 1] (layers/attention.py:127-133)
    const int slot = p < 0 ? 0 : (p >= a.max_seq ? a.max_seq - 1 : p);
    bf16* dst = (is_v ? a.vc : a.kc) + (((size_t)b * a.max_seq + slot) * a.nkv + kvh) * a.hd;
    dst[d0] = __float2bfloat16_rn(x1);
    dst[d1] = __float2bfloat16_rn(x2);
  }
}

__device__ __forceinline__ void qkv_store(const GemvArgs& a, int g, int m, float acc0, float acc1) {
  float b0, b1;
  qkv_bias_pair(a, g, b0, b1);
  qkv_store_b(a, g, m, acc0, acc1, b0, b1, a.pos, a.inv_freq);
}

// gate/up packing (jsx_pack_gate_up): group j holds rows (gate_j, up_j).
// models/glm4.py:47-49 with jax.nn.silu(x) = x * sigmoid(x) on bf16 arrays.
__device__ __forceinline__ void swiglu_store(const GemvArgs& a, int g, int m, float acc0, float acc1) {
  const float gate = rbf(acc0);
  const float up = rbf(acc1);
  const float sig = rbf(1.0f / (1.0f + expf(-gate)));
  const float act = rbf(rbf(gate * sig) * up);
  a.y[(size_t)m * (a.N >> 1) + g] = __float2bfloat16_rn(act);
}

template <int M>
__device__ __forceinline__ void epi_qkv(const GemvArgs& a, int g, const float (&acc)[kRows][M],
                                        int lane) {
  if (lane >= M) return;
  qkv_store(a, g, lane, pick<M>(acc, 0, lane), pick<M>(acc, 1, lane));
}

template <int M>
__device__ __forceinline__ void epi_swiglu(const GemvArgs& a, int g, const float (&acc)[kRows][M],
                                           int lane) {
  if (lane >= M) return;
  swiglu_store(a, g, lane, pick<M>(acc, 0, lane), pick<M>(acc, 1, lane));
}

// Epilogue of one row pair (packed rows 2g, 2g+1) for token m; returns the
// argmax key of the pair (LM head) or 0.
template <int EPI>
__device__ __forceinline__ unsigned long long epi_pair(const GemvArgs& a, const CommDev& c, bool multi,
                                                       uint32_t epoch, int g, int m, float v0, float v1) {
  const int r0 = 2 * g;
  if constexpr (EPI == EPI_LINEAR) {
    float y0 = rbf(v0), y1 = rbf(v1);
    if (a.bias) {
      y0 = rbf(y0 + ldbf(a.bias + r0));
      y1 = rbf(y1 + ldbf(a.bias + r0 + 1));
    }
    a.y[(size_t)m * a.N + r0] = __float2bfloat16_rn(y0);
    a.y[(size_t)m * a.N + r0 + 1] = __float2bfloat16_rn(y1);
  } else if constexpr (EPI == EPI_QKV) {
    qkv_store(a, g, m, v0, v1);
  } else if constexpr (EPI == EPI_SWIGLU) {
    swiglu_store(a, g, m, v0, v1);
  } else if constexpr (EPI == EPI_ROWAR) {
    if (a.addend) {
      v0 += ldbf(a.addend + (size_t)m * a.N + r0);
      v1 += ldbf(a.addend + (size_t)m * a.N + r0 + 1);
    }
    if (!multi) {
      bf16* hp = a.h + (size_t)m * a.N + r0;
      hp[0] = __float2bfloat16_rn(__bfloat162float(hp[0]) + rbf(v0));
      hp[1] = __float2bfloat16_rn(__bfloat162float(hp[1]) + rbf(v1));
    } else {
      for (int d = 0; d < c.world; ++d) {
        unsigned long long* dst = data_ptr(c, d, epoch & 1, c.rank, m) + r0;
        ll_put(dst, v0, epoch);
        ll_put(dst + 1, v1, epoch);
      }
    }
  } else if constexpr (EPI == EPI_LMHEAD) {
    const float l0 = rbf(v0), l1 = rbf(v1);
    if (a.y) {
      a.y[(size_t)m * a.N + r0] = __float2bfloat16_rn(l0);
      a.y[(size_t)m * a.N + r0 + 1] = __float2bfloat16_rn(l1);
    }
    const unsigned long long k0 = argmax_key(l0, (uint32_t)(a.vocab_offset + r0));
    const unsigned long long k1 = argmax_key(l1, (uint32_t)(a.vocab_offset + r0 + 1));
    return k0 > k1 ? k0 : k1;
  }
  return 0ull;
}

}  // namespace jsx
