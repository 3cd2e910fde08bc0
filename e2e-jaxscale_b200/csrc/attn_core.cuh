// Split-context GQA decode attention: the per-item body shared by the
// standalone kernel (attention.cu) and the whole-step decode kernel.
#pragma once

#include <math.h>

#include "common.cuh"
#include "launch.cuh"

namespace jsx {

constexpr int kChunk = 64;                 // cache rows per split
constexpr int kRowBlocks = kChunk / 32;    // 32-row blocks per split (one row per lane)
constexpr int kAttnThreads = 128;

// Work unit ("item"): one split of kChunk cache rows of one (sequence, kv head)
// for a group of gi query heads of that kv head (hg = G / gi groups).  Splitting
// the G heads of a kv head over several items spreads a decode step's small
// attention over more CTAs and lets several CTAs merge splits in parallel.
struct AttnArgs {
  const bf16* q;   // [B][nq][hd]
  const bf16* kc;  // [B][max_seq][nkv][hd]
  const bf16* vc;
  bf16* out;       // [B][nq*hd]
  const int32_t* pos;
  int B, nq, nkv, hd, max_seq, splits;
  int gi, hg;      // heads per item, head groups per kv head
  float scale;
  float* part;     // [B*nkv*hg][splits][split_stride(gi)]: acc [gi][hd], then m [gi], l [gi] (padded)
  uint32_t* cnt;   // [B*nkv*hg], zero on entry, left zero
  uint64_t* trace; // null, or 8 %globaltimer stamps of group 0: item (0, 0) start, staged,
                   // scores, softmax, P.V done, completion counted; the group's merge done,
                   // the group's merge start (its last split counted)
  int no_merge;    // items only write their split records; the consumer merges them
                   // (whole-step kernel, small groups: the o_proj staging)
  uint32_t* dist_err;  // null, or the distributed merge (every split item merges a share
                       // of the group's heads once all have counted; needs every item of
                       // the launch on its own co-resident CTA) and its error word, set
                       // when the wait for the other splits gives up
};

constexpr long long kMergeWaitCycles = 4000000000ll;  // ~2 s at the 1965 MHz max clock

__device__ __forceinline__ void attn_stamp(const AttnArgs& a, int vb, int s, int k) {
  if (a.trace != nullptr && vb == 0 && (s == 0 || k >= 6) && threadIdx.x == 0) a.trace[k] = globaltimer();
}

// floats per split record: the accumulator tile, then (m, l) per head, padded so
// every record starts on a 16-byte boundary (float4 reads in the combine)
__host__ __device__ __forceinline__ int split_stride(int G, int hd) {
  return G * hd + ((2 * G + 3) & ~3);
}

__host__ __device__ __forceinline__ int attn_heads_per_item(int G) {
  return G % 4 == 0 ? 4 : (G % 2 == 0 ? 2 : 1);
}

// Workspace: 256-byte header, per-item-group counters padded to 256 bytes, then
// the split records.
struct AttnLayout {
  int gi, hg, splits, stride;
  size_t counter_bytes;  // header + counters (must be zero before a call)
  size_t bytes;          // whole workspace
};

// Heads are split over several items only when (sequence, kv head, split)
// items alone would leave most of the GPU idle (small batches): each head
// group re-reads the kv head's rows.
__host__ __device__ __forceinline__ AttnLayout attn_layout(int B, int nq, int nkv, int hd, int max_seq) {
  AttnLayout L;
  const int G = nq / nkv;
  L.splits = (max_seq + kChunk - 1) / kChunk;
  L.gi = ((size_t)B * nkv * L.splits >= 256) ? G : attn_heads_per_item(G);
  L.hg = G / L.gi;
  L.stride = split_stride(L.gi, hd);
  const size_t groups = (size_t)B * nkv * L.hg;
  L.counter_bytes = 256 + ((groups * sizeof(uint32_t) + 255) & ~(size_t)255);
  L.bytes = L.counter_bytes + groups * L.splits * L.stride * sizeof(float);
  return L;
}

// Tensor-core item shape: a group of 16 query heads (the MMA's M) with
// head_dim 128 (GLM-4: 32 query heads over 2 kv heads).  Shared rows are padded
// to 136 bf16 (272 bytes) so the 8 row addresses of an ldmatrix hit distinct banks.
constexpr int kMmaHeads = 16;
constexpr int kMmaHd = 128;
constexpr int kRowPad = kMmaHd + 8;   // bf16 per q/K/V row in shared memory
constexpr int kPPad = kChunk + 8;     // bf16 per probability row
__host__ __device__ __forceinline__ bool attn_use_mma(int gi, int hd) {
  return gi >= 1 && gi <= kMmaHeads && hd == kMmaHd;
}

// Shared bytes of one item: q (fp32), scores/probabilities, padded K rows, V
// rows; the combine reuses the K/V area.  Tensor-core items: q, K, V (bf16,
// padded rows), fp32 scores, bf16 probabilities; the combine reuses all but q.
__host__ __device__ __forceinline__ size_t attn_smem(int gi, int hd, int splits) {
  const size_t combine = ((size_t)2 * splits * gi + 2 * gi) * 4;
  if (attn_use_mma(gi, hd)) {
    const size_t work = (size_t)2 * kChunk * kRowPad * 2 + (size_t)kMmaHeads * kChunk * 4 +
                        (size_t)kMmaHeads * kPPad * 2;
    return (size_t)kMmaHeads * kRowPad * 2 + (work > combine ? work : combine);
  }
  const int hw = hd / 2;
  const size_t stage = (size_t)kChunk * (hw + 1) * 4 + (size_t)2 * kChunk * hw * 4;
  return (size_t)gi * hd * 4 + (size_t)gi * kChunk * 4 + (stage > combine ? stage : combine);
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
// 16-byte global -> shared copy; src_bytes < 16 zero-fills the rest (0: no read)
__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ uint32_t dyn_smem_bytes() {
  uint32_t r;
  asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(r));
  return r;
}

// Distributed completion (a.dist_err): every split item of group vb counts
// itself, waits (bounded) until all have, then merges heads s, s + splits, ...
// of the group, with the arithmetic of the shared-memory merge in attn_finish
// (per head: warp max of m, warp sum of l * exp(m - M), weights exp(m - M) / L;
// per output pair a sequential FMA over the splits).  While warp 0 forms a
// head's weights, the other warps have that head's accumulators of the first
// kSeg splits in flight to shared memory (cp.async), so the merge costs one L2
// round trip after the wait, on every split CTA at once instead of all heads on
// the last one.  The counter rises to splits (arrivals), then to 2 splits
// (merges done); the last merge leaves it zero for the next use, which follows
// a grid barrier.  Needs the tensor-core item's shared memory past `scratch`
// (>= 41 KB): (splits + 3) / 4 * 16 + kSeg * hd * 4 + splits * 4 bytes.
__device__ __forceinline__ uint32_t attn_ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

constexpr int kSeg = 32;  // splits of one head staged at a time by the distributed merge

template <int NT>
__device__ __forceinline__ void attn_finish_distributed(const AttnArgs& a, int vb, int s, int b, int head0,
                                                        int cur, float* scratch) {
  const int gi = a.gi, hd = a.hd, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int stride = split_stride(gi, hd);
  __threadfence();
  __syncthreads();
  if (tid == 0 && atomicAdd(a.cnt + vb, 1u) != (uint32_t)a.splits - 1u) {  // the last arrival does not wait
    const long long t0 = clock64();
    uint32_t it = 0;
    while (attn_ld_acquire(a.cnt + vb) < (uint32_t)a.splits) {
      if ((++it & 63u) == 0 && clock64() - t0 > kMergeWaitCycles) {
        atomicOr(a.dist_err, 2u);
        break;
      }
    }
  }
  if (tid == 0) __threadfence();  // the other splits' records are read after this point
  __syncthreads();
  attn_stamp(a, vb, s, 5);
  attn_stamp(a, vb, s, 7);
  const int used = (cur + kChunk) / kChunk;
  const float* pb = a.part + (size_t)vb * a.splits * stride;
  bf16* ob = a.out + ((size_t)b * a.nq + head0) * hd;
  float* w = scratch;                        // [used] m, then the weights of the head being merged
  float* os = scratch + ((used + 3) & ~3);   // [kSeg][hd] its accumulators, kSeg splits at a time
  float* lw = os + kSeg * hd;                // [used] l
  const int d2 = tid - 32, nd2 = hd >> 1, n16 = hd >> 2;
  for (int h = s; h < gi; h += a.splits) {
    float2 o = make_float2(0.f, 0.f);
    for (int t0 = 0; t0 < used; t0 += kSeg) {
      const int nt = used - t0 < kSeg ? used - t0 : kSeg;
      if (tid >= 32) {
        for (int i = tid - 32; i < nt * n16; i += NT - 32) {
          const int t = i / n16, c = i - t * n16;
          cp_async16(os + t * hd + 4 * c, pb + (size_t)(t0 + t) * stride + h * hd + 4 * c, 16u);
        }
      }
      if (t0 == 0 && warp == 0) {
        // m and l of every split in one round trip, then as in the shared-memory merge
        float M = -INFINITY;
        for (int t = lane; t < used; t += 32) {
          const float m = __ldcg(pb + (size_t)t * stride + gi * hd + h);
          lw[t] = __ldcg(pb + (size_t)t * stride + gi * hd + gi + h);
          w[t] = m;
          M = fmaxf(M, m);
        }
        M = warp_max(M);
        float L = 0.f;
        for (int t = lane; t < used; t += 32) {
          const float e = expf(w[t] - M);
          w[t] = e;
          L = fmaf(lw[t], e, L);
        }
        L = warp_sum(L);
        for (int t = lane; t < used; t += 32) w[t] = w[t] / L;
      }
      cp_async_wait_all();
      __syncthreads();
      if (d2 >= 0 && d2 < nd2) {
        const float2* o2 = reinterpret_cast<const float2*>(os) + d2;
        for (int t = 0; t < nt; ++t) {
          const float wt = w[t0 + t];
          const float2 v = o2[t * nd2];
          o.x = fmaf(v.x, wt, o.x);
          o.y = fmaf(v.y, wt, o.y);
        }
      }
      __syncthreads();  // os (and, after the last segment, w) are reused
    }
    if (d2 >= 0 && d2 < nd2) *reinterpret_cast<uint32_t*>(ob + h * hd + 2 * d2) = pack2(o.x, o.y);
  }
  attn_stamp(a, vb, 0, 6);
  if (tid == 0 && atomicAdd(a.cnt + vb, 1u) == 2u * (uint32_t)a.splits - 1u) a.cnt[vb] = 0u;
}

// Completion of one item: the item that completes the set of splits of group
// vb merges them (flash-decoding combine).  Weights w_t[h] = exp(m_t - M) / L
// are formed once in shared memory (`scratch`, free once the item's own work is
// done), then every output element is a short dot product over the splits.
// When the used split records fit in the dynamic shared memory past `scratch`
// they arrive there in one cp.async round trip (m, l and the accumulators
// together) and the merge runs from shared memory; otherwise m and l are read
// first and the accumulators streamed from L2.
template <int NT>
__device__ __forceinline__ void attn_finish(const AttnArgs& a, int vb, int s, int b, int head0, int cur,
                                            float* scratch) {
  __shared__ bool is_last;
  extern __shared__ __align__(16) unsigned char attn_dyn_smem[];
  const int gi = a.gi, hd = a.hd, tid = threadIdx.x;
  const int stride = split_stride(gi, hd);
  // the next kernel may launch once every item has reached this point (only
  // the merges remain), not earlier: its CTAs would take SMs from later items
  pdl_launch_dependents();
  if (a.no_merge) return;  // the records are merged by their consumer after a grid barrier
  if (a.dist_err != nullptr) {
    attn_finish_distributed<NT>(a, vb, s, b, head0, cur, scratch);
    return;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) is_last = atomicAdd(a.cnt + vb, 1u) == (uint32_t)(a.splits - 1);
  __syncthreads();
  attn_stamp(a, vb, s, 5);
  if (!is_last) return;
  __threadfence();
  attn_stamp(a, vb, s, 7);

  const int used = (cur + kChunk) / kChunk;
  const float* pb = a.part + (size_t)vb * a.splits * stride;
  bf16* ob = a.out + ((size_t)b * a.nq + head0) * hd;
  const uint32_t off = smem_addr(scratch) - smem_addr(attn_dyn_smem);
  const size_t need = ((size_t)used * stride + (size_t)used * gi) * 4;
  if ((off & 15u) == 0 && (hd & 1) == 0 && off + need <= dyn_smem_bytes()) {
    constexpr int NW = NT / 32;
    const int lane = tid & 31, warp = tid >> 5;
    float* rec = scratch;                        // [used][stride]: the records as stored
    float* w = rec + (size_t)used * stride;      // [used][gi] weights
    const int n16 = (used * stride) >> 2;        // stride is a multiple of 4
    for (int i = tid; i < n16; i += NT) cp_async16(rec + 4 * i, pb + 4 * i, 16u);
    cp_async_wait_all();
    __syncthreads();
    for (int h = warp; h < gi; h += NW) {
      float M = -INFINITY;
      for (int t = lane; t < used; t += 32) M = fmaxf(M, rec[(size_t)t * stride + gi * hd + h]);
      M = warp_max(M);
      float L = 0.f;
      for (int t = lane; t < used; t += 32) {
        const float e = expf(rec[(size_t)t * stride + gi * hd + h] - M);
        w[t * gi + h] = e;
        L = fmaf(rec[(size_t)t * stride + gi * hd + gi + h], e, L);
      }
      L = warp_sum(L);
      for (int t = lane; t < used; t += 32) w[t * gi + h] = w[t * gi + h] / L;
    }
    __syncthreads();
    const int nv = (gi * hd) >> 1, s2 = stride >> 1;
    const float2* r2 = reinterpret_cast<const float2*>(rec);
    for (int i = tid; i < nv; i += NT) {
      const int h = (i << 1) / hd;
      float2 o = make_float2(0.f, 0.f);
      for (int t = 0; t < used; ++t) {
        const float wt = w[t * gi + h];
        const float2 v = r2[(size_t)t * s2 + i];
        o.x = fmaf(v.x, wt, o.x);
        o.y = fmaf(v.y, wt, o.y);
      }
      *reinterpret_cast<uint32_t*>(ob + (i << 1)) = pack2(o.x, o.y);
    }
    if (tid == 0) a.cnt[vb] = 0u;
    attn_stamp(a, vb, 0, 6);
    return;
  }
  float* wm = scratch;                       // [used][gi] m, then weights
  float* wl = wm + a.splits * gi;            // [used][gi] l
  float* Mg = wl + a.splits * gi;            // [gi]
  float* Lg = Mg + gi;                       // [gi]
  for (int i = tid; i < used * gi; i += NT) {
    const int t = i / gi, h = i - (i / gi) * gi;
    wm[i] = __ldcg(pb + (size_t)t * stride + gi * hd + h);
    wl[i] = __ldcg(pb + (size_t)t * stride + gi * hd + gi + h);
  }
  __syncthreads();
  for (int h = tid; h < gi; h += NT) {
    float M = -INFINITY;
    for (int t = 0; t < used; ++t) M = fmaxf(M, wm[t * gi + h]);
    float L = 0.f;
    for (int t = 0; t < used; ++t) L = fmaf(wl[t * gi + h], expf(wm[t * gi + h] - M), L);
    Mg[h] = M;
    Lg[h] = L;
  }
  __syncthreads();
  for (int i = tid; i < used * gi; i += NT) {
    const int h = i - (i / gi) * gi;
    wm[i] = expf(wm[i] - Mg[h]) / Lg[h];
  }
  __syncthreads();
  const int nv = (gi * hd) >> 2;
  for (int i = tid; i < nv; i += NT) {
    const int e = i << 2, h = e / hd;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
    for (int t = 0; t < used; ++t) {
      const float w = wm[t * gi + h];
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
  if (tid == 0) a.cnt[vb] = 0u;
  attn_stamp(a, vb, 0, 6);
}

// One work item: cache rows [64 s, 64 s + 64) of item group vb (sequence b,
// kv head kvh, head group j; vb = (b * nkv + kvh) * hg + j), processed by NT
// threads; the item that completes the set of splits of its group merges them.
// kCoherent: read q and the cache with ld.global.cg (they were written by
// other CTAs of the same kernel).  kEager: load the split's rows together with
// the position (one round trip; splits past the context load rows they do not
// use) instead of after it.
template <int NT, bool kCoherent, bool kEager>
__device__ __forceinline__ void attn_item(const AttnArgs& a, int s, int vb, unsigned char* smem_raw) {
  constexpr int NW = NT / 32;
  const int G = a.nq / a.nkv, gi = a.gi;
  const int hd = a.hd, hw = hd >> 1, hq = hd >> 3;  // head dim in 4- and 16-byte words
  const int stride = split_stride(gi, hd);
  float* qs = reinterpret_cast<float*>(smem_raw);                  // [gi][hd]
  float* ps = qs + gi * hd;                                         // [gi][kChunk]
  uint32_t* ks = reinterpret_cast<uint32_t*>(ps + gi * kChunk);     // [kChunk][hw+1] (padded)
  uint32_t* vs = ks + kChunk * (hw + 1);                            // [kChunk][hw]

  const int b = vb / (a.nkv * a.hg);
  const int kvh = (vb / a.hg) % a.nkv, j = vb % a.hg;
  const int head0 = kvh * G + j * gi;  // first query head of the item
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __syncthreads();  // a CTA may run several items back to back over the same shared memory
  attn_stamp(a, vb, s, 0);

  // q, the item's K/V rows and the position are loaded together: the rows are
  // staged whether or not they are inside the context (masked below)
  const int p0 = s * kChunk;
  int cur = a.pos[b];
  const int rows = kEager ? min(kChunk, a.max_seq - p0) : max(0, min(kChunk, min(cur, a.max_seq - 1) + 1 - p0));
  const bf16* qg = a.q + ((size_t)b * a.nq + head0) * hd;
  for (int i = tid; i < gi * hd; i += NT) qs[i] = __bfloat162float(kCoherent ? __ldcg(qg + i) : qg[i]);
  const size_t row_stride = (size_t)a.nkv * hd;  // elements between consecutive cache rows
  const bf16* kb = a.kc + ((size_t)b * a.max_seq + p0) * row_stride + (size_t)kvh * hd;
  const bf16* vbp = a.vc + ((size_t)b * a.max_seq + p0) * row_stride + (size_t)kvh * hd;
  // K and V rows arrive by cp.async (cp.async.cg reads through L2: coherent
  // with other CTAs' writes), every copy of the thread in flight at once; K
  // lands unpadded in kraw and each thread repacks its own chunks into the
  // padded rows the score loop reads.
  uint32_t* kraw = vs + kChunk * hw;  // [kChunk][hw]
  for (int i = tid; i < rows * hq; i += NT) {
    const int r = i / hq, c = i - (i / hq) * hq;
    cp_async16(kraw + r * hw + 4 * c, kb + (size_t)r * row_stride + 8 * c, 16u);
    cp_async16(vs + r * hw + 4 * c, vbp + (size_t)r * row_stride + 8 * c, 16u);
  }
  cp_async_wait_all();
  for (int i = tid; i < rows * hq; i += NT) {
    const int r = i / hq, c = i - (i / hq) * hq;
    const uint4 kv = *reinterpret_cast<const uint4*>(kraw + r * hw + 4 * c);
    uint32_t* kd = ks + r * (hw + 1) + 4 * c;
    kd[0] = kv.x; kd[1] = kv.y; kd[2] = kv.z; kd[3] = kv.w;
  }
  if (cur > a.max_seq - 1) cur = a.max_seq - 1;
  if (cur < 0) cur = 0;
  int n = cur + 1 - p0;  // rows of this split inside [0, cur]; n <= rows
  if (n > kChunk) n = kChunk;
  float* part = a.part + ((size_t)vb * a.splits + s) * stride;
  __syncthreads();
  attn_stamp(a, vb, s, 1);

  if (n > 0) {
    // scores: one (head, 32-row block) task per warp pass, one row per lane;
    // q is a broadcast read, four partial sums keep the FMA chains short
    for (int t = warp; t < gi * kRowBlocks; t += NW) {
      const int h = t / kRowBlocks, r = (t - h * kRowBlocks) * 32 + lane;
      const float* qr = qs + h * hd;
      const uint32_t* kr = ks + r * (hw + 1);
      float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll 4
      for (int w = 0; w < hw; w += 2) {
        const uint32_t k0 = kr[w], k1 = kr[w + 1];
        d0 = fmaf(qr[2 * w], bf_lo(k0), d0);
        d1 = fmaf(qr[2 * w + 1], bf_hi(k0), d1);
        d2 = fmaf(qr[2 * w + 2], bf_lo(k1), d2);
        d3 = fmaf(qr[2 * w + 3], bf_hi(k1), d3);
      }
      ps[h * kChunk + r] = r < n ? ((d0 + d1) + (d2 + d3)) * a.scale : -INFINITY;
    }
    __syncthreads();
    attn_stamp(a, vb, s, 2);
    // softmax pieces of the split: per head max m, e = exp(s - m), sum l
    for (int h = warp; h < gi; h += NW) {
      float v[kRowBlocks];
      float m = -INFINITY;
#pragma unroll
      for (int rb = 0; rb < kRowBlocks; ++rb) {
        v[rb] = ps[h * kChunk + rb * 32 + lane];
        m = fmaxf(m, v[rb]);
      }
      m = warp_max(m);
      float l = 0.f;
#pragma unroll
      for (int rb = 0; rb < kRowBlocks; ++rb) {
        const float e = (rb * 32 + lane < n) ? expf(v[rb] - m) : 0.f;
        ps[h * kChunk + rb * 32 + lane] = e;
        l += e;
      }
      l = warp_sum(l);
      if (lane == 0) {
        part[gi * hd + h] = m;
        part[gi * hd + gi + h] = l;
      }
    }
    __syncthreads();
    attn_stamp(a, vb, s, 3);
    // P.V: each thread owns up to 4 (head, dim-pair) outputs and walks the rows
    // once for all of them (independent accumulators)
    for (int base = tid; base < gi * hw; base += 4 * NT) {
      float x0[4], x1[4];
      int gg[4], ww[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int i = base + k * NT;
        gg[k] = i < gi * hw ? i / hw : 0;
        ww[k] = i < gi * hw ? i - (i / hw) * hw : 0;
        x0[k] = 0.f;
        x1[k] = 0.f;
      }
#pragma unroll 2
      for (int p = 0; p < n; ++p) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t vw = vs[p * hw + ww[k]];
          const float pr = ps[gg[k] * kChunk + p];
          x0[k] = fmaf(pr, bf_lo(vw), x0[k]);
          x1[k] = fmaf(pr, bf_hi(vw), x1[k]);
        }
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int i = base + k * NT;
        if (i < gi * hw) {
          part[gg[k] * hd + 2 * ww[k]] = x0[k];
          part[gg[k] * hd + 2 * ww[k] + 1] = x1[k];
        }
      }
    }
  }

  attn_stamp(a, vb, s, 4);
  attn_finish<NT>(a, vb, s, b, head0, cur, reinterpret_cast<float*>(ks));
}

// ---- tensor-core item (mma.sync m16n8k16, bf16 in, fp32 accumulate) ----------
// S = Q K^T and O = P V are m16n8k16 MMAs with the item's query heads as M (a
// group of gi <= 16 heads, padded with zero rows to 16): every K/V element is
// read from shared memory once per item instead of once per head and output as
// in the CUDA-core form (which measured 7 us of shared-memory-bound compute per
// 64-row item at 4 heads).  The probabilities enter P.V rounded to bf16 (the
// reference also rounds them to bf16 before its P.V product); m and l stay fp32.
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Staging of an item's cache rows ahead of the grid barrier that publishes this
// step's q and its new K/V row (whole-step kernel): the rows of split s that
// earlier steps wrote (before the position cur) are copied into the item's
// shared-memory rows, rows past cur are zero-filled, the row at cur is left for
// attn_item_mma<..., kPre = true>, which copies it and q after the barrier.
// Returns the clamped position.  The positions do not change during a step.
template <int NT>
__device__ __forceinline__ int attn_prefetch_mma(const AttnArgs& a, int s, int vb, unsigned char* smem_raw) {
  bf16* ks = reinterpret_cast<bf16*>(smem_raw) + kMmaHeads * kRowPad;
  bf16* vs = ks + kChunk * kRowPad;
  const int b = vb / (a.nkv * a.hg), kvh = (vb / a.hg) % a.nkv;
  const int p0 = s * kChunk;
  int cur = a.pos[b];
  if (cur > a.max_seq - 1) cur = a.max_seq - 1;
  if (cur < 0) cur = 0;
  const int rc = cur - p0;  // row of position cur in this split (may lie outside it)
  const size_t row_stride = (size_t)a.nkv * kMmaHd;
  const bf16* kb = a.kc + ((size_t)b * a.max_seq + p0) * row_stride + (size_t)kvh * kMmaHd;
  const bf16* vbp = a.vc + ((size_t)b * a.max_seq + p0) * row_stride + (size_t)kvh * kMmaHd;
  for (int i = threadIdx.x; i < kChunk * 16; i += NT) {
    const int r = i >> 4, c = i & 15;
    if (r == rc) continue;
    const bool live = r < rc;
    const size_t off = (size_t)(live ? r : 0) * row_stride + c * 8;
    cp_async16(ks + r * kRowPad + c * 8, kb + off, live ? 16u : 0u);
    cp_async16(vs + r * kRowPad + c * 8, vbp + off, live ? 16u : 0u);
  }
  return cur;
}

template <int NT, bool kCoherent, bool kEager, bool kPre = false>
__device__ __forceinline__ void attn_item_mma(const AttnArgs& a, int s, int vb, unsigned char* smem_raw,
                                              int pre_cur = 0) {
  constexpr int NW = NT / 32;
  constexpr int RW = kChunk / NW;   // score rows per warp (16 or 8)
  constexpr int NS = RW / 8;        // n8 score tiles per warp
  constexpr int DW = kMmaHd / NW;   // output dims per warp (32 or 16)
  constexpr int NO = DW / 8;        // n8 output tiles per warp
  static_assert(NW == 4 || NW == 8, "4 or 8 warps");
  const int G = a.nq / a.nkv, gi = a.gi;
  const int stride = split_stride(gi, kMmaHd);
  bf16* qs = reinterpret_cast<bf16*>(smem_raw);  // [16][kRowPad], rows >= gi zero
  bf16* ks = qs + kMmaHeads * kRowPad;            // [64][kRowPad]
  bf16* vs = ks + kChunk * kRowPad;               // [64][kRowPad]
  float* ss = reinterpret_cast<float*>(vs + kChunk * kRowPad);  // [16][64] scores
  bf16* ps = reinterpret_cast<bf16*>(ss + kMmaHeads * kChunk);  // [16][kPPad] probabilities

  const int b = vb / (a.nkv * a.hg);
  const int kvh = (vb / a.hg) % a.nkv, j = vb % a.hg;
  const int head0 = kvh * G + j * gi;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __syncthreads();  // a CTA may run several items back to back over the same shared memory
  attn_stamp(a, vb, s, 0);

  const int p0 = s * kChunk;
  int cur = kPre ? pre_cur : a.pos[b];
  const int rows = kEager ? min(kChunk, a.max_seq - p0) : max(0, min(kChunk, min(cur, a.max_seq - 1) + 1 - p0));
  if (cur > a.max_seq - 1) cur = a.max_seq - 1;
  if (cur < 0) cur = 0;
  int n = cur + 1 - p0;  // rows of this split inside [0, cur]
  if (n > kChunk) n = kChunk;
  // q, K and V arrive by cp.async (cp.async.cg reads through L2: coherent with
  // other CTAs' writes), every copy of the thread in flight at once.  Rows past
  // the staged ones are zero-filled; with eager staging the rows at or past n
  // are zeroed after the copies land (masked probabilities are exactly 0 and
  // must not meet non-finite cache contents).
  const bf16* qg = a.q + ((size_t)b * a.nq + head0) * kMmaHd;
  for (int i = tid; i < kMmaHeads * 16; i += NT) {
    const int h = i >> 4, c = i & 15;
    cp_async16(qs + h * kRowPad + c * 8, qg + (h < gi ? h : 0) * kMmaHd + c * 8, h < gi ? 16u : 0u);
  }
  const size_t row_stride = (size_t)a.nkv * kMmaHd;
  const bf16* kb = a.kc + ((size_t)b * a.max_seq + p0) * row_stride + (size_t)kvh * kMmaHd;
  const bf16* vbp = a.vc + ((size_t)b * a.max_seq + p0) * row_stride + (size_t)kvh * kMmaHd;
  if (kPre) {
    // every other row is in flight since attn_prefetch_mma
    const int rc = cur - p0;
    if (rc >= 0 && rc < kChunk && tid < 16) {
      const size_t off = (size_t)rc * row_stride + tid * 8;
      cp_async16(ks + rc * kRowPad + tid * 8, kb + off, 16u);
      cp_async16(vs + rc * kRowPad + tid * 8, vbp + off, 16u);
    }
  } else {
    const int live_rows = kEager ? rows : min(rows, n);
    for (int i = tid; i < kChunk * 16; i += NT) {
      const int r = i >> 4, c = i & 15;
      const bool live = r < live_rows;
      const size_t off = (size_t)(live ? r : 0) * row_stride + c * 8;
      cp_async16(ks + r * kRowPad + c * 8, kb + off, live ? 16u : 0u);
      cp_async16(vs + r * kRowPad + c * 8, vbp + off, live ? 16u : 0u);
    }
  }
  cp_async_wait_all();
  if (kEager && !kPre) {
    for (int i = tid; i < kChunk * 16; i += NT) {
      const int r = i >> 4, c = i & 15;
      if (r >= n && r < rows) {
        *reinterpret_cast<uint4*>(ks + r * kRowPad + c * 8) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(vs + r * kRowPad + c * 8) = make_uint4(0, 0, 0, 0);
      }
    }
  }
  float* part = a.part + ((size_t)vb * a.splits + s) * stride;
  __syncthreads();
  attn_stamp(a, vb, s, 1);

  if (n > 0) {
    const int g = lane >> 2, t4 = lane & 3;
    // S = Q K^T for rows [RW warp, RW warp + RW)
    float sc[NS][4];
#pragma unroll
    for (int jn = 0; jn < NS; ++jn) sc[jn][0] = sc[jn][1] = sc[jn][2] = sc[jn][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < kMmaHd / 16; ++kk) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4(smem_addr(qs + (lane & 15) * kRowPad + 16 * kk + (lane >> 4) * 8), a0, a1, a2, a3);
#pragma unroll
      for (int jn = 0; jn < NS; ++jn) {
        uint32_t b0, b1;
        ldsm_x2(smem_addr(ks + (RW * warp + 8 * jn + (lane & 7)) * kRowPad + 16 * kk + ((lane >> 3) & 1) * 8),
                b0, b1);
        mma_bf16_16816(sc[jn], a0, a1, a2, a3, b0, b1);
      }
    }
#pragma unroll
    for (int jn = 0; jn < NS; ++jn) {
      const int r = RW * warp + 8 * jn + 2 * t4;
      ss[g * kChunk + r] = r < n ? sc[jn][0] * a.scale : -INFINITY;
      ss[g * kChunk + r + 1] = r + 1 < n ? sc[jn][1] * a.scale : -INFINITY;
      ss[(g + 8) * kChunk + r] = r < n ? sc[jn][2] * a.scale : -INFINITY;
      ss[(g + 8) * kChunk + r + 1] = r + 1 < n ? sc[jn][3] * a.scale : -INFINITY;
    }
    __syncthreads();
    attn_stamp(a, vb, s, 2);
    // softmax pieces per head: m, e = exp(s - m) (bf16 for the MMA), l (fp32)
    for (int h = warp; h < gi; h += NW) {
      float v[kRowBlocks];
      float m = -INFINITY;
#pragma unroll
      for (int rb = 0; rb < kRowBlocks; ++rb) {
        v[rb] = ss[h * kChunk + rb * 32 + lane];
        m = fmaxf(m, v[rb]);
      }
      m = warp_max(m);
      float l = 0.f;
#pragma unroll
      for (int rb = 0; rb < kRowBlocks; ++rb) {
        const float e = (rb * 32 + lane < n) ? expf(v[rb] - m) : 0.f;
        ps[h * kPPad + rb * 32 + lane] = __float2bfloat16_rn(e);
        l += e;
      }
      l = warp_sum(l);
      if (lane == 0) {
        part[gi * kMmaHd + h] = m;
        part[gi * kMmaHd + gi + h] = l;
      }
    }
    __syncthreads();
    attn_stamp(a, vb, s, 3);
    // O = P V for dims [DW warp, DW warp + DW)
    float o[NO][4];
#pragma unroll
    for (int jn = 0; jn < NO; ++jn) o[jn][0] = o[jn][1] = o[jn][2] = o[jn][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < kChunk / 16; ++kk) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4(smem_addr(ps + (lane & 15) * kPPad + 16 * kk + (lane >> 4) * 8), a0, a1, a2, a3);
#pragma unroll
      for (int jn = 0; jn < NO; ++jn) {
        uint32_t b0, b1;
        ldsm_x2_t(smem_addr(vs + (16 * kk + (lane & 7) + ((lane >> 3) & 1) * 8) * kRowPad + DW * warp + 8 * jn),
                  b0, b1);
        mma_bf16_16816(o[jn], a0, a1, a2, a3, b0, b1);
      }
    }
#pragma unroll
    for (int jn = 0; jn < NO; ++jn) {
      const int d = DW * warp + 8 * jn + 2 * t4;
      if (g < gi) *reinterpret_cast<float2*>(part + g * kMmaHd + d) = make_float2(o[jn][0], o[jn][1]);
      if (g + 8 < gi) *reinterpret_cast<float2*>(part + (g + 8) * kMmaHd + d) = make_float2(o[jn][2], o[jn][3]);
    }
  }
  attn_stamp(a, vb, s, 4);
  attn_finish<NT>(a, vb, s, b, head0, cur, reinterpret_cast<float*>(ks));
}

// The item body for the group shape: tensor-core form for head_dim 128 (groups
// of up to 16 heads), CUDA-core form otherwise.
template <int NT, bool kCoherent, bool kEager>
__device__ __forceinline__ void attn_item_any(const AttnArgs& a, int s, int vb, unsigned char* smem_raw) {
  if (attn_use_mma(a.gi, a.hd)) attn_item_mma<NT, kCoherent, kEager>(a, s, vb, smem_raw);
  else attn_item<NT, kCoherent, kEager>(a, s, vb, smem_raw);
}

}  // namespace jsx
