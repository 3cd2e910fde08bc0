// Sampling of the next token (runner.py:315-359, _jit_sample): repetition
// penalty -> temperature -> top-k -> top-p on the k candidates -> categorical.
//
// One CTA of 1024 threads per sequence; thread t owns the contiguous vocabulary
// slice [t * chunk, (t + 1) * chunk), so index order is thread order.
//   values   v = bf16(x / rp) or bf16(x * rp) where the token is present (x > 0
//            divides), then bf16(v / T); rp and T are rounded to bf16 first, as
//            the reference's Python scalars are when they meet a bf16 array;
//   top-k    radix select on the 16-bit order key of v: a histogram of the high
//            byte finds the byte of the k-th largest key, a histogram of the low
//            byte inside it the exact key; every larger key is a candidate, and
//            of the keys equal to it the lowest indices (a block scan of per-thread
//            tie counts gives each tie its rank in index order), like lax.top_k;
//            the k candidates are sorted by (value desc, index asc) (bitonic sort);
//   top-p    fp32 softmax over the k sorted values, running sum in order; a
//            candidate whose preceding mass reaches top_p gets bf16(-1e9);
//   draw     argmax over candidates of bf16(value + g), g the caller's Gumbel
//            noise for the k candidates in that order (jax.random.categorical
//            draws the same form from its own generator); first maximum wins.
#include <math.h>

#include "common.cuh"
#include "launch.cuh"

namespace jsx {

constexpr int kSampleThreads = 1024;
constexpr int kSampleMaxK = 256;

struct SampleArgs {
  const bf16* logits;       // [B][V]
  const uint8_t* presence;  // [B][V] or null
  const bf16* gumbel;       // [B][k]
  int32_t* tokens;          // [B]
  int V, k, chunk;
  float rp, temp;           // already bf16-rounded; temp 1 = none
  float top_p;
};

__device__ __forceinline__ uint32_t order_key16(float v) {
  const uint32_t u = __float_as_uint(v) >> 16;  // v is a bf16 value
  return (u & 0x8000u) ? (~u & 0xffffu) : (u | 0x8000u);
}

__device__ __forceinline__ float sample_value(const SampleArgs& a, const bf16* lg, const uint8_t* pr, int i) {
  float x = __bfloat162float(lg[i]);
  if (pr && pr[i]) x = rbf(x > 0.f ? x / a.rp : x * a.rp);
  if (a.temp != 1.f) x = rbf(x / a.temp);
  return x;
}

// exclusive prefix sum over the block's threads (1024), total in *total
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = warp_sums[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    warp_sums[lane] = w;  // inclusive
    if (lane == 31) *total = w;
  }
  __syncthreads();
  return x - v + (warp > 0 ? warp_sums[warp - 1] : 0);
}

__global__ void __launch_bounds__(kSampleThreads) k_sample(SampleArgs a) {
  __shared__ int hist[256];
  __shared__ int warp_sums[32];
  __shared__ int sel[4];  // high byte, low byte, keys above the threshold, candidates
  __shared__ int total;
  __shared__ unsigned long long cand[kSampleMaxK];
  pdl_wait();  // the logits come from the previous kernel
  const int b = blockIdx.x, tid = threadIdx.x;
  const bf16* lg = a.logits + (size_t)b * a.V;
  const uint8_t* pr = a.presence ? a.presence + (size_t)b * a.V : nullptr;
  const int i0 = tid * a.chunk, i1 = min(a.V, i0 + a.chunk);

  // ---- radix select of the k-th largest key: high byte ----
  for (int j = tid; j < 256; j += kSampleThreads) hist[j] = 0;
  __syncthreads();
  for (int i = i0; i < i1; ++i) atomicAdd(&hist[order_key16(sample_value(a, lg, pr, i)) >> 8], 1);
  __syncthreads();
  if (tid == 0) {
    int above = 0, bin = 255;
    for (; bin > 0; --bin) {
      if (above + hist[bin] >= a.k) break;
      above += hist[bin];
    }
    sel[0] = bin;
    sel[2] = above;  // keys with a larger high byte
  }
  __syncthreads();
  const uint32_t hi = (uint32_t)sel[0];
  for (int j = tid; j < 256; j += kSampleThreads) hist[j] = 0;
  __syncthreads();
  // ---- low byte inside the selected high byte ----
  for (int i = i0; i < i1; ++i) {
    const uint32_t key = order_key16(sample_value(a, lg, pr, i));
    if ((key >> 8) == hi) atomicAdd(&hist[key & 0xffu], 1);
  }
  __syncthreads();
  if (tid == 0) {
    int above = sel[2], bin = 255;
    for (; bin > 0; --bin) {
      if (above + hist[bin] >= a.k) break;
      above += hist[bin];
    }
    sel[1] = bin;
    sel[2] = above;  // keys above the threshold key
    sel[3] = 0;
  }
  __syncthreads();
  const uint32_t thr = (hi << 8) | (uint32_t)sel[1];
  const int need_eq = a.k - sel[2];
  // ---- candidates: every key above the threshold, the lowest-index ties ----
  int nt = 0;
  for (int i = i0; i < i1; ++i) nt += order_key16(sample_value(a, lg, pr, i)) == thr;
  const int tie0 = block_exclusive_scan(nt, warp_sums, &total);
  for (int j = tid; j < kSampleMaxK; j += kSampleThreads) cand[j] = 0ull;
  __syncthreads();
  int rank = tie0;
  for (int i = i0; i < i1; ++i) {
    const float v = sample_value(a, lg, pr, i);
    const uint32_t key = order_key16(v);
    bool take = key > thr;
    if (key == thr) take = rank++ < need_eq;
    if (take) {
      const int slot = atomicAdd(&sel[3], 1);
      if (slot < kSampleMaxK)
        cand[slot] = ((unsigned long long)key << 32) | (unsigned long long)(0xffffffffu - (uint32_t)i);
    }
  }
  __syncthreads();
  // ---- sort the candidates: larger key first, then lower index ----
  for (int size = 2; size <= kSampleMaxK; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      if (tid < kSampleMaxK) {
        const int j = tid ^ stride;
        if (j > tid) {
          const bool desc = (tid & size) == 0;
          const unsigned long long x = cand[tid], y = cand[j];
          if ((x < y) == desc) {
            cand[tid] = y;
            cand[j] = x;
          }
        }
      }
      __syncthreads();
    }
  }
  // ---- top-p and the draw (k <= 256 values, one thread) ----
  if (tid == 0) {
    const int k = a.k;
    const float neg = rbf(-1e9f);
    auto value_of = [&](int j) {
      const uint32_t key = (uint32_t)(cand[j] >> 32);
      const uint32_t u = (key & 0x8000u) ? (key & 0x7fffu) : (~key & 0xffffu);
      return __uint_as_float(u << 16);
    };
    float mx = value_of(0), sum = 0.f;
    if (a.top_p < 1.f)
      for (int j = 0; j < k; ++j) sum += expf(value_of(j) - mx);
    float cum = 0.f, best = -INFINITY;
    int best_j = 0;
    const bf16* g = a.gumbel + (size_t)b * k;
    for (int j = 0; j < k; ++j) {
      float v = value_of(j);
      if (a.top_p < 1.f) {
        const float p = expf(v - mx) / sum;
        cum += p;
        if (cum - p >= a.top_p) v = neg;
      }
      const float z = rbf(v + __bfloat162float(g[j]));
      if (z > best) {
        best = z;
        best_j = j;
      }
    }
    a.tokens[b] = (int32_t)(0xffffffffu - (uint32_t)(cand[best_j] & 0xffffffffull));
  }
}

}  // namespace jsx

using namespace jsx;

extern "C" int jsx_sample(const void* logits, const uint8_t* presence, const void* gumbel, int32_t* tokens_out, int B,
                          int V, float repetition_penalty, float temperature, int top_k, float top_p, void* stream) {
  JSX_REQUIRE(logits && gumbel && tokens_out, "null pointer argument");
  const int k = top_k > 0 ? top_k : 200;
  JSX_REQUIRE(B >= 1 && V >= 1 && k <= kSampleMaxK && k <= V, "B=%d V=%d k=%d (k <= min(256, V))", B, V, k);
  JSX_REQUIRE(repetition_penalty > 0.f && temperature > 0.f && top_p > 0.f, "penalty, temperature and top_p must be > 0");
  SampleArgs a;
  a.logits = (const bf16*)logits;
  a.presence = presence;
  a.gumbel = (const bf16*)gumbel;
  a.tokens = tokens_out;
  a.V = V;
  a.k = k;
  a.chunk = (V + kSampleThreads - 1) / kSampleThreads;
  a.rp = __bfloat162float(__float2bfloat16_rn(repetition_penalty));
  a.temp = temperature == 1.f ? 1.f : __bfloat162float(__float2bfloat16_rn(temperature));
  a.top_p = top_p;
  JSX_CUDA(launch_kernel(k_sample, dim3(B), dim3(kSampleThreads), 0, (cudaStream_t)stream, a));
  return JSX_OK;
}
