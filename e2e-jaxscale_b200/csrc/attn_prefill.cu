// Causal prefill attention over the static KV cache (layers/attention.py:101-160
// with the prefill mask of runner.py:26-32): the S query tokens of every
// sequence, at positions start .. start + S - 1, attend to cache rows
// [0, position] of their sequence (rows before `start` hold an earlier prefix,
// rows from `start` were written by this prefill's q/k/v projection).
//
// One CTA = 64 query rows of one query head (4 warps x 16 rows); the kv head's
// cache rows stream through shared memory in blocks of 64 keys (cp.async,
// double-buffered).  Per block: S = Q K^T on mma.sync m16n8k16 (bf16 in, fp32
// accumulate), causal mask, online softmax in fp32 (running max and sum per
// row), P rounded to bf16 and O += P V on the same MMA; O / l at the end.
// Attention is 2 x 2 x hd flops per (query, key) pair, about 2 % of a GLM-4
// prefill's flops at 1024 tokens, so the legacy MMA is enough here; the
// projections around it run on tcgen05 (tc_wide.cu).
//
// CTAs with the longest key ranges (the last query blocks) are scheduled first.
#include "attn_core.cuh"
#include "common.cuh"
#include "launch.cuh"

namespace jsx {

constexpr int kPfRows = 64;     // query rows per CTA
constexpr int kPfKeys = 64;     // keys per block
constexpr int kPfHd = 128;      // head_dim of the MMA path
constexpr int kPfPad = kPfHd + 8;
constexpr int kPfThreads = 128;
constexpr size_t kPfSmem = (size_t)(kPfRows + 4 * kPfKeys) * kPfPad * 2;  // Q, 2 x K, 2 x V

struct PfArgs {
  const bf16* q;   // [B * S][nq * 128]
  const bf16* kc;  // [B][max_seq][nkv][128]
  const bf16* vc;
  bf16* out;       // [B * S][nq * 128]
  int B, S, start, nq, nkv, max_seq;
  float scale_log2;  // head_dim^-0.5 x log2(e)
};

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) { return pack2(lo, hi); }

__global__ void __launch_bounds__(kPfThreads, 2) k_attn_prefill(PfArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  bf16* qs = reinterpret_cast<bf16*>(smem);   // [64][kPfPad]
  bf16* ks = qs + kPfRows * kPfPad;            // [2][64][kPfPad]
  bf16* vs = ks + 2 * kPfKeys * kPfPad;        // [2][64][kPfPad]
  const int qb = gridDim.x - 1 - blockIdx.x;   // longest key ranges first
  const int h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (a.nq / a.nkv);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t4 = lane & 3;
  const int i0 = qb * kPfRows;
  const int last = min(i0 + kPfRows, a.S) - 1;  // last query row of the block
  const int kend = a.start + last + 1;          // keys [0, kend)
  const int nkb = (kend + kPfKeys - 1) / kPfKeys;
  const size_t qstride = (size_t)a.nq * kPfHd;
  const size_t rs = (size_t)a.nkv * kPfHd;
  // q and the new cache rows come from the previous kernel (launched with
  // programmatic dependent launch, it may still be running)
  pdl_wait();

  const bf16* qg = a.q + (size_t)(b * a.S + i0) * qstride + h * kPfHd;
  for (int e = tid; e < kPfRows * 16; e += kPfThreads) {
    const int r = e >> 4, c = e & 15;
    const bool live = i0 + r < a.S;
    cp_async16(qs + r * kPfPad + c * 8, qg + (size_t)(live ? r : 0) * qstride + c * 8, live ? 16u : 0u);
  }
  const bf16* kbase = a.kc + (size_t)b * a.max_seq * rs + kvh * kPfHd;
  const bf16* vbase = a.vc + (size_t)b * a.max_seq * rs + kvh * kPfHd;
  auto load_kv = [&](int kb, int buf) {
    bf16* kd = ks + buf * kPfKeys * kPfPad;
    bf16* vd = vs + buf * kPfKeys * kPfPad;
    for (int e = tid; e < kPfKeys * 16; e += kPfThreads) {
      const int r = e >> 4, c = e & 15;
      const int key = kb * kPfKeys + r;
      const bool live = key < kend;
      const size_t off = (size_t)(live ? key : 0) * rs + c * 8;
      cp_async16(kd + r * kPfPad + c * 8, kbase + off, live ? 16u : 0u);
      cp_async16(vd + r * kPfPad + c * 8, vbase + off, live ? 16u : 0u);
    }
  };
  load_kv(0, 0);
  cp_async_commit();

  // running state of rows g and g + 8 of this warp's 16
  float o[kPfHd / 8][4];
#pragma unroll
  for (int j = 0; j < kPfHd / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  uint32_t qa[kPfHd / 16][4];
  const int qrow0 = a.start + i0 + warp * 16 + g;  // query positions of rows g and g + 8

  for (int kb = 0; kb < nkb; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 < nkb) {
      load_kv(kb + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait_group<1>();
    } else {
      cp_async_wait_group<0>();
    }
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int kk = 0; kk < kPfHd / 16; ++kk)
        ldsm_x4(smem_addr(qs + (warp * 16 + (lane & 15)) * kPfPad + 16 * kk + (lane >> 4) * 8), qa[kk][0], qa[kk][1],
                qa[kk][2], qa[kk][3]);
    }
    const bf16* kt = ks + buf * kPfKeys * kPfPad;
    const bf16* vt = vs + buf * kPfKeys * kPfPad;
    // S = Q K^T, 16 x 64 per warp
    float sc[kPfKeys / 8][4];
#pragma unroll
    for (int jn = 0; jn < kPfKeys / 8; ++jn) sc[jn][0] = sc[jn][1] = sc[jn][2] = sc[jn][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < kPfHd / 16; ++kk) {
#pragma unroll
      for (int jn = 0; jn < kPfKeys / 8; ++jn) {
        uint32_t b0, b1;
        ldsm_x2(smem_addr(kt + (8 * jn + (lane & 7)) * kPfPad + 16 * kk + ((lane >> 3) & 1) * 8), b0, b1);
        mma_bf16_16816(sc[jn], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
      }
    }
    // scale (log2 domain), causal mask, running max
    float mx[2] = {mrow[0], mrow[1]};
#pragma unroll
    for (int jn = 0; jn < kPfKeys / 8; ++jn) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = kb * kPfKeys + 8 * jn + 2 * t4 + (e & 1);
        const int qp = qrow0 + (e >> 1) * 8;
        const float s = key <= qp ? sc[jn][e] * a.scale_log2 : -INFINITY;
        sc[jn][e] = s;
        mx[e >> 1] = fmaxf(mx[e >> 1], s);
      }
    }
    float alpha[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      // key 0 is visible to every row, so the running max is finite from block 0 on
      alpha[r] = exp2f(mrow[r] - mx[r]);
      mrow[r] = mx[r];
      lrow[r] *= alpha[r];
    }
#pragma unroll
    for (int j = 0; j < kPfHd / 8; ++j) {
      o[j][0] *= alpha[0];
      o[j][1] *= alpha[0];
      o[j][2] *= alpha[1];
      o[j][3] *= alpha[1];
    }
    // P = exp2(S - m) (fp32 sums, bf16 into the MMA), O += P V
#pragma unroll
    for (int kk = 0; kk < kPfKeys / 16; ++kk) {
      float p[2][4];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float v = exp2f(sc[2 * kk + half][e] - mrow[e >> 1]);
          p[half][e] = v;
          lrow[e >> 1] += v;
        }
      }
      const uint32_t a0 = pack_bf2(p[0][0], p[0][1]);
      const uint32_t a1 = pack_bf2(p[0][2], p[0][3]);
      const uint32_t a2 = pack_bf2(p[1][0], p[1][1]);
      const uint32_t a3 = pack_bf2(p[1][2], p[1][3]);
#pragma unroll
      for (int jd = 0; jd < kPfHd / 8; ++jd) {
        uint32_t b0, b1;
        ldsm_x2_t(smem_addr(vt + (16 * kk + (lane & 7) + ((lane >> 3) & 1) * 8) * kPfPad + 8 * jd), b0, b1);
        mma_bf16_16816(o[jd], a0, a1, a2, a3, b0, b1);
      }
    }
    __syncthreads();  // the buffer is refilled by the next iteration's prefetch
  }

  float inv[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    float l = lrow[r];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    inv[r] = 1.f / l;
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int i = i0 + warp * 16 + g + 8 * r;
    if (i >= a.S) continue;
    bf16* orow = a.out + (size_t)(b * a.S + i) * qstride + h * kPfHd;
#pragma unroll
    for (int jd = 0; jd < kPfHd / 8; ++jd)
      *reinterpret_cast<uint32_t*>(orow + 8 * jd + 2 * t4) =
          pack2(o[jd][2 * r] * inv[r], o[jd][2 * r + 1] * inv[r]);
  }
}

}  // namespace jsx

using namespace jsx;

extern "C" int jsx_attn_prefill(const void* q, const void* k_cache, const void* v_cache, void* out, int B, int S,
                                int start_pos, int nq, int nkv, int head_dim, int max_seq, float scale,
                                void* stream) {
  JSX_REQUIRE(q && k_cache && v_cache && out, "null pointer argument");
  JSX_REQUIRE(B >= 1 && B <= 65535 && S >= 1 && nq >= 1 && nq <= 65535 && nkv >= 1 && nq % nkv == 0,
              "B=%d S=%d nq=%d nkv=%d", B, S, nq, nkv);
  JSX_REQUIRE(start_pos >= 0 && (long long)start_pos + S <= max_seq, "start_pos=%d S=%d max_seq=%d", start_pos, S,
              max_seq);
  JSX_REQUIRE(aligned16(q) && aligned16(k_cache) && aligned16(v_cache) && aligned16(out),
              "tensors must be 16-byte aligned");
  if (head_dim != kPfHd) {
    set_error("jsx_attn_prefill: head_dim=%d (the kernel takes 128)", head_dim);
    return JSX_ENOTSUP;
  }
  PfArgs a;
  a.q = (const bf16*)q;
  a.kc = (const bf16*)k_cache;
  a.vc = (const bf16*)v_cache;
  a.out = (bf16*)out;
  a.B = B; a.S = S; a.start = start_pos; a.nq = nq; a.nkv = nkv; a.max_seq = max_seq;
  a.scale_log2 = scale * 1.4426950408889634f;
  JSX_CUDA(cudaFuncSetAttribute(k_attn_prefill, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPfSmem));
  const dim3 grid((S + kPfRows - 1) / kPfRows, nq, B);
  JSX_CUDA(launch_kernel(k_attn_prefill, grid, dim3(kPfThreads), kPfSmem, (cudaStream_t)stream, a));
  return JSX_OK;
}
