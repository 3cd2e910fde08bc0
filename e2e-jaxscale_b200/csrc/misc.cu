// Small kernels of the decode path: weight packing (load time), standalone
// RMSNorm, embedding gather, MoE router.
#include <math.h>

#include "common.cuh"
#include "launch.cuh"

namespace jsx {

// ---- packing -------------------------------------------------------------------
// Output row R of a packed matrix [R_total][K] is column col(R) of one of up to
// three source matrices [K][ld].  32x32 shared-memory tiles keep both the read
// (along the source columns) and the write (along K) coalesced.
enum PackMode { PACK_T = 0, PACK_QKV = 1, PACK_GU = 2 };

struct PackArgs {
  const bf16* src[3];
  int ld[3];
  bf16* dst;
  int K, R;
  int mode;
  int nq, nkv, hd, rot;
};

__device__ __forceinline__ void pack_source(const PackArgs& a, int R, int& which, int& col) {
  if (a.mode == PACK_T) {
    which = 0;
    col = R;
  } else if (a.mode == PACK_GU) {
    which = R & 1;  // rows (gate_j, up_j)
    col = R >> 1;
  } else {
    const int g = R >> 1, second = R & 1;
    const int gph = a.hd >> 1, rh = a.rot >> 1;
    const int head = g / gph, j = g - head * gph;
    int d;
    if (j < rh) d = second ? j + rh : j;
    else d = a.rot + 2 * (j - rh) + second;
    if (head < a.nq) { which = 0; col = head * a.hd + d; }
    else if (head < a.nq + a.nkv) { which = 1; col = (head - a.nq) * a.hd + d; }
    else { which = 2; col = (head - a.nq - a.nkv) * a.hd + d; }
  }
}

__global__ void k_pack(PackArgs a) {
  __shared__ bf16 tile[32][33];
  pdl_wait();  // the source may come from the previous kernel
  const int R0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  for (int i = ty; i < 32; i += 8) {
    const int R = R0 + tx, k = k0 + i;
    if (R < a.R && k < a.K) {
      int which, col;
      pack_source(a, R, which, col);
      tile[i][tx] = a.src[which][(size_t)k * a.ld[which] + col];
    }
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int R = R0 + i, k = k0 + tx;
    if (R < a.R && k < a.K) a.dst[(size_t)R * a.K + k] = tile[tx][i];
  }
}

static int run_pack(const PackArgs& a, cudaStream_t s) {
  dim3 grid((a.R + 31) / 32, (a.K + 31) / 32);
  k_pack<<<grid, dim3(32, 8), 0, s>>>(a);
  JSX_LAUNCHED("k_pack");
  return JSX_OK;
}

// ---- RMSNorm (layers/normalization.py:31-37) --------------------------------------
__global__ void k_rmsnorm(const bf16* __restrict__ x, const bf16* __restrict__ g, bf16* __restrict__ y,
                          int hidden, float eps) {
  __shared__ float red[32];
  const bf16* xr = x + (size_t)blockIdx.x * hidden;
  bf16* yr = y + (size_t)blockIdx.x * hidden;
  pdl_wait();
  float ss = 0.f;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    const float f = __bfloat162float(xr[i]);
    ss = fmaf(f, f, ss);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = 1.0f / sqrtf(t / (float)hidden + eps);
  }
  __syncthreads();
  const float r = red[0];
  for (int i = threadIdx.x; i < hidden; i += blockDim.x)
    yr[i] = __float2bfloat16_rn((__bfloat162float(xr[i]) * r) * __bfloat162float(g[i]));
}

// Vectorised form for hidden % 8 == 0 and 16-byte aligned rows: one CTA of 128
// threads per row, the row held in registers (up to kNormVec 16-byte vectors
// per thread, hidden <= 128 * 8 * kNormVec), so x and gamma cross the memory
// system once.  Same per-element formula as k_rmsnorm.
constexpr int kNormThreads = 128;
constexpr int kNormVec = 8;
__global__ void __launch_bounds__(kNormThreads) k_rmsnorm_vec(const bf16* __restrict__ x,
                                                              const bf16* __restrict__ g,
                                                              bf16* __restrict__ y, int hidden, float eps) {
  __shared__ float red[kNormThreads / 32];
  const int nvec = hidden >> 3;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)blockIdx.x * hidden);
  const uint4* gv = reinterpret_cast<const uint4*>(g);
  uint4* yr = reinterpret_cast<uint4*>(y + (size_t)blockIdx.x * hidden);
  pdl_wait();
  pdl_launch_dependents();
  uint4 xv[kNormVec], gw[kNormVec];
#pragma unroll
  for (int j = 0; j < kNormVec; ++j) {
    const int v = threadIdx.x + j * kNormThreads;
    xv[j] = v < nvec ? xr[v] : make_uint4(0, 0, 0, 0);
    gw[j] = v < nvec ? gv[v] : make_uint4(0, 0, 0, 0);
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kNormVec; ++j) {
    float f[8];
    unpack8(xv[j], f);
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(f[e], f[e], ss);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) t += red[w];
  const float r = 1.0f / sqrtf(t / (float)hidden + eps);
#pragma unroll
  for (int j = 0; j < kNormVec; ++j) {
    const int v = threadIdx.x + j * kNormThreads;
    if (v < nvec) {
      float f[8], q[8];
      unpack8(xv[j], f);
      unpack8(gw[j], q);
      uint4 o;
      o.x = pack2((f[0] * r) * q[0], (f[1] * r) * q[1]);
      o.y = pack2((f[2] * r) * q[2], (f[3] * r) * q[3]);
      o.z = pack2((f[4] * r) * q[4], (f[5] * r) * q[5]);
      o.w = pack2((f[6] * r) * q[6], (f[7] * r) * q[7]);
      yr[v] = o;
    }
  }
}

// ---- embedding (layers/embedding.py:35-51) -----------------------------------------
// jnp.take's default out-of-bounds mode fills with NaN; the same happens here
// (no out-of-range read).
__global__ void k_embed(const int32_t* __restrict__ ids, const bf16* __restrict__ table,
                        bf16* __restrict__ out, int hidden, int vocab) {
  pdl_wait();
  pdl_launch_dependents();
  const int id = ids[blockIdx.x];
  bf16* o = out + (size_t)blockIdx.x * hidden;
  if (id < 0 || id >= vocab) {
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) o[i] = __float2bfloat16_rn(NAN);
    return;
  }
  const bf16* t = table + (size_t)id * hidden;
  if ((hidden & 7) == 0) {
    const uint4* tv = reinterpret_cast<const uint4*>(t);
    uint4* ov = reinterpret_cast<uint4*>(o);
    for (int i = threadIdx.x; i < (hidden >> 3); i += blockDim.x) ov[i] = tv[i];
  } else {
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) o[i] = t[i];
  }
}

// ---- MoE router (layers/moe.py:54-79) ------------------------------------------------
constexpr int kGateMaxE = 256;
constexpr int kGateMaxK = 8;

__global__ void k_moe_gate(const bf16* __restrict__ x, const bf16* __restrict__ w, const float* bias,
                           bf16* __restrict__ topk_w, int32_t* __restrict__ topk_i, int H, int E,
                           int k, float scale, int norm) {
  __shared__ float logits[kGateMaxE];
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  pdl_wait();
  if (w == nullptr) {
    // logits given directly: x is [N][E] bf16
    for (int e = threadIdx.x; e < E; e += blockDim.x)
      logits[e] = __bfloat162float(x[(size_t)t * E + e]);
  } else {
    const bf16* xr = x + (size_t)t * H;
    for (int e = warp; e < E; e += nw) {
      const bf16* wr = w + (size_t)e * H;
      float acc = 0.f;
      for (int i = lane; i < H; i += 32) acc = fmaf(__bfloat162float(xr[i]), __bfloat162float(wr[i]), acc);
      acc = warp_sum(acc);
      if (lane == 0) logits[e] = rbf(acc);  // bf16 logits (params dtype), then f32
    }
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  // f32 softmax (jax.nn.softmax: exp(x - max) / sum)
  float mx = -INFINITY;
  for (int e = 0; e < E; ++e) mx = fmaxf(mx, logits[e]);
  float sum = 0.f;
  for (int e = 0; e < E; ++e) {
    logits[e] = expf(logits[e] - mx);
    sum += logits[e];
  }
  for (int e = 0; e < E; ++e) logits[e] = logits[e] / sum;  // scores
  // top-k on corrected scores; ties -> lower index first (lax.top_k)
  int sel[kGateMaxK];
  float wsum = 0.f;
  for (int j = 0; j < k; ++j) {
    int bi = -1;
    float bv = -INFINITY;
    for (int e = 0; e < E; ++e) {
      bool taken = false;
      for (int q = 0; q < j; ++q) taken |= (sel[q] == e);
      if (taken) continue;
      const float v = logits[e] + (bias ? bias[e] : 0.f);
      if (bi < 0 || v > bv) { bv = v; bi = e; }
    }
    sel[j] = bi;
    wsum += logits[bi];
  }
  for (int j = 0; j < k; ++j) {
    float v = logits[sel[j]];
    if (norm) v = v / (wsum + 1e-20f);
    v = v * scale;
    topk_w[(size_t)t * k + j] = __float2bfloat16_rn(v);
    topk_i[(size_t)t * k + j] = sel[j];
  }
}

}  // namespace jsx

using namespace jsx;

extern "C" int jsx_pack_transpose(const void* w_kn, void* w_nk, int K, int N, void* stream) {
  JSX_REQUIRE(w_kn && w_nk && K >= 1 && N >= 1, "bad transpose arguments");
  PackArgs a = {};
  a.src[0] = (const bf16*)w_kn; a.ld[0] = N; a.dst = (bf16*)w_nk; a.K = K; a.R = N; a.mode = PACK_T;
  return run_pack(a, (cudaStream_t)stream);
}

extern "C" int jsx_pack_qkv(const void* w_q, const void* w_k, const void* w_v, void* w_qkv, int K,
                            int nq, int nkv, int head_dim, int rotary_dim, void* stream) {
  JSX_REQUIRE(w_q && w_k && w_v && w_qkv && K >= 1 && nq >= 1 && nkv >= 1, "bad qkv arguments");
  JSX_REQUIRE(head_dim % 2 == 0 && rotary_dim % 2 == 0 && rotary_dim <= head_dim,
              "head_dim=%d rotary_dim=%d", head_dim, rotary_dim);
  PackArgs a = {};
  a.src[0] = (const bf16*)w_q; a.ld[0] = nq * head_dim;
  a.src[1] = (const bf16*)w_k; a.ld[1] = nkv * head_dim;
  a.src[2] = (const bf16*)w_v; a.ld[2] = nkv * head_dim;
  a.dst = (bf16*)w_qkv; a.K = K; a.R = (nq + 2 * nkv) * head_dim; a.mode = PACK_QKV;
  a.nq = nq; a.nkv = nkv; a.hd = head_dim; a.rot = rotary_dim;
  return run_pack(a, (cudaStream_t)stream);
}

extern "C" int jsx_pack_gate_up(const void* w_gate, const void* w_up, void* w_gu, int K, int I,
                                void* stream) {
  JSX_REQUIRE(w_gate && w_up && w_gu && K >= 1 && I >= 1, "bad gate/up arguments");
  PackArgs a = {};
  a.src[0] = (const bf16*)w_gate; a.ld[0] = I;
  a.src[1] = (const bf16*)w_up; a.ld[1] = I;
  a.dst = (bf16*)w_gu; a.K = K; a.R = 2 * I; a.mode = PACK_GU;
  return run_pack(a, (cudaStream_t)stream);
}

extern "C" int jsx_rmsnorm(const void* x, const void* gamma, void* y, int rows, int hidden, float eps,
                           void* stream) {
  JSX_REQUIRE(x && gamma && y && rows >= 1 && hidden >= 1, "bad rmsnorm arguments");
  if (hidden % 8 == 0 && hidden <= kNormThreads * 8 * kNormVec && aligned16(x) && aligned16(gamma) &&
      aligned16(y)) {
    JSX_CUDA(launch_kernel(k_rmsnorm_vec, dim3(rows), dim3(kNormThreads), 0, (cudaStream_t)stream,
                           (const bf16*)x, (const bf16*)gamma, (bf16*)y, hidden, eps));
    return JSX_OK;
  }
  JSX_CUDA(launch_kernel(k_rmsnorm, dim3(rows), dim3(256), 0, (cudaStream_t)stream,
                         (const bf16*)x, (const bf16*)gamma, (bf16*)y, hidden, eps));
  return JSX_OK;
}

extern "C" int jsx_embed(const int32_t* ids, const void* table, void* out, int M, int hidden,
                         int vocab, void* stream) {
  JSX_REQUIRE(ids && table && out && M >= 1 && hidden >= 1 && vocab >= 1, "bad embed arguments");
  JSX_REQUIRE((hidden & 7) != 0 || (aligned16(table) && aligned16(out)),
              "table/out must be 16-byte aligned");
  JSX_CUDA(launch_kernel(k_embed, dim3(M), dim3(128), 0, (cudaStream_t)stream, ids,
                         (const bf16*)table, (bf16*)out, hidden, vocab));
  return JSX_OK;
}

extern "C" int jsx_moe_gate(const void* x, const void* w_nk, const float* correction_bias,
                            void* topk_w, int32_t* topk_idx, int N, int H, int E, int k, float scale,
                            int norm, void* stream) {
  JSX_REQUIRE(x && topk_w && topk_idx, "null pointer argument");
  JSX_REQUIRE(N >= 1 && E >= 1 && E <= kGateMaxE && k >= 1 && k <= kGateMaxK && k <= E,
              "N=%d E=%d k=%d outside the router limits (E<=%d, k<=%d)", N, E, k, kGateMaxE, kGateMaxK);
  JSX_REQUIRE(w_nk == nullptr || H >= 1, "H=%d", H);
  JSX_CUDA(launch_kernel(k_moe_gate, dim3(N), dim3(256), 0, (cudaStream_t)stream, (const bf16*)x,
                         (const bf16*)w_nk, correction_bias, (bf16*)topk_w, topk_idx, H, E, k, scale,
                         norm));
  return JSX_OK;
}
