// Batch-1 decode kernels for Whisper-large-v3-turbo on B200 (sm_100a).
//
// The reference decode step (custom/model.py:107-123) is 46 launches: its own LayerNorm,
// split/combine attention, LM-head argmax and finalize kernels around 24 cuBLAS GEMVs, a GELU and
// two index_selects. Here the step is 34 launches chained with programmatic dependent launch
// (PDL):
//
//   per layer: ln_gemv(QKV, LN1 [+embed on layer 0]) -> attention(self, fused cache write and
//              in-kernel split combine) -> gemv_residual(out) -> ln_gemv(cross q, LN2)
//              -> attention(cross) -> gemv_residual(cross out) -> ln_gemv(fc1 + GELU, LN3)
//              -> gemv_residual(fc2)
//   then:      lm_head(final LN + GEMV + argmax + finalize)
//
// Every kernel is HBM-streaming: the weight rows (or K/V rows) a CTA needs are requested with
// bulk async copies into shared memory *before* griddepcontrol.wait, so the weight stream of
// kernel N overlaps the tail of kernel N-1. Dot products use the same per-lane order and warp
// xor-tree as the reference kernels so that the LM-head logits, LayerNorm outputs and attention
// outputs are bit-identical to the reference kernels given identical inputs.
#include <cooperative_groups.h>

#include <mutex>

#include "fw_common.cuh"
#include "fw_host.h"

namespace fw {

namespace cg = cooperative_groups;

FW_DEFINE_ERROR_WORD();

__device__ __forceinline__ void flag_error(unsigned bits) { atomicOr(&g_fw_dev_error, bits); }

// ---------------------------------------------------------------------------------------------
// Block-level synchronisation of the 256 compute threads. Stand-alone kernels use __syncthreads;
// the persistent decode kernel (which also runs a producer warp that never joins) uses named
// barrier 1 over exactly the 256 compute threads.
template <bool kNamed>
__device__ __forceinline__ void compute_sync() {
  if (kNamed)
    asm volatile("bar.sync 1, 256;" ::: "memory");
  else
    __syncthreads();
}

// LayerNorm over 1280 values held 5 per thread by a 256-thread block (index tid + 256*i).
// Summation order matches add_layernorm_kernel (custom/kernels/whisper_kernels.cu:217-267):
// per-thread running sums, warp xor-tree, then the eight warp partials in order.
template <bool kNamed = false>
__device__ __forceinline__ void ln1280_stats(const float (&v)[5], float* red, float eps, float& mean, float& inv) {
  // red: 16 floats, [0, 8) warp sums, [8, 16) warp sums of squares. The caller separates two calls
  // with a barrier of its own.
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < 5; ++i) sum += v[i];
  sum = warp_sum(sum);
  if (lane == 0) red[warp] = sum;
  compute_sync<kNamed>();
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) m += red[i];
  m /= static_cast<float>(kHidden);
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < 5; ++i) {
    const float d = v[i] - m;
    sq = fmaf(d, d, sq);
  }
  sq = warp_sum(sq);
  if (lane == 0) red[8 + warp] = sq;
  compute_sync<kNamed>();
  float var = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) var += red[8 + i];
  mean = m;
  inv = rsqrtf(var / static_cast<float>(kHidden) + eps);
}

__device__ __forceinline__ float ln_apply(float v, float mean, float inv, float g, float b) {
  return fmaf((v - mean) * inv, g, b);
}

// Dot product of one 1280-wide fp16 row (16-byte chunks lane + 32*c) with x held as 40 floats per
// lane in the same chunk order. The fma order is the reference LM-head order (whisper_kernels.cu:58-68).
__device__ __forceinline__ float dot1280_lane(const uint4* row, const float (&xf)[40]) {
  float acc = 0.f;
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int c = 0; c < 5; ++c) {
    const uint4 wv = row[lane + 32 * c];
    const half2* p = reinterpret_cast<const half2*>(&wv);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __half22float2(p[k]);
      acc = fmaf(f.x, xf[c * 8 + 2 * k], acc);
      acc = fmaf(f.y, xf[c * 8 + 2 * k + 1], acc);
    }
  }
  return acc;
}

// kRows dot products of 1280-wide fp16 rows `stride` elements apart with x (as dot1280_lane), their
// loads and fma chains interleaved, followed by the warp xor-tree of each: every result is
// bit-identical to warp_sum(dot1280_lane(row, xf)), only the latency overlaps.
template <int kRows>
__device__ __forceinline__ void dot1280_rows(const half* row0, int stride, const float (&xf)[40], float (&out)[kRows]) {
  const int lane = threadIdx.x & 31;
  float acc[kRows];
#pragma unroll
  for (int r = 0; r < kRows; ++r) acc[r] = 0.f;
#pragma unroll
  for (int c = 0; c < 5; ++c) {
    uint4 wv[kRows];
#pragma unroll
    for (int r = 0; r < kRows; ++r) wv[r] = reinterpret_cast<const uint4*>(row0 + r * stride)[lane + 32 * c];
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      const half2* p = reinterpret_cast<const half2*>(&wv[r]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(p[k]);
        acc[r] = fmaf(f.x, xf[c * 8 + 2 * k], acc[r]);
        acc[r] = fmaf(f.y, xf[c * 8 + 2 * k + 1], acc[r]);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int r = 0; r < kRows; ++r) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
#pragma unroll
  for (int r = 0; r < kRows; ++r) out[r] = acc[r];
}

__device__ __forceinline__ void load_x40(const half* xs, float (&xf)[40]) {
  const int lane = threadIdx.x & 31;
  const uint4* x4 = reinterpret_cast<const uint4*>(xs);
#pragma unroll
  for (int c = 0; c < 5; ++c) {
    const uint4 v = x4[lane + 32 * c];
    const half2* p = reinterpret_cast<const half2*>(&v);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __half22float2(p[k]);
      xf[c * 8 + 2 * k] = f.x;
      xf[c * 8 + 2 * k + 1] = f.y;
    }
  }
}

// ---------------------------------------------------------------------------------------------
// add_layernorm (reference surface).
__global__ void __launch_bounds__(256) add_layernorm_kernel(half* __restrict__ h, const half* __restrict__ x,
                                                            const half* __restrict__ gamma,
                                                            const half* __restrict__ beta, half* __restrict__ y,
                                                            float eps) {
  __shared__ float red[16];
  pdl_wait();
  pdl_trigger();
  float v[5];
#pragma unroll
  for (int i = 0; i < 5; ++i) {
    const int idx = threadIdx.x + i * 256;
    float r = __half2float(h[idx]);
    if (x) {
      r = round_half(r + __half2float(x[idx]));
      h[idx] = __float2half(r);
    }
    v[i] = r;
  }
  float mean, inv;
  ln1280_stats(v, red, eps, mean, inv);
#pragma unroll
  for (int i = 0; i < 5; ++i) {
    const int idx = threadIdx.x + i * 256;
    y[idx] = __float2half(ln_apply(v[i], mean, inv, __half2float(gamma[idx]), __half2float(beta[idx])));
  }
}

// ---------------------------------------------------------------------------------------------
// Split-K single-query attention. CTA (head, split) owns 64 keys; the 64 K rows and 64 V rows are
// bulk-copied into shared memory before griddepcontrol.wait (cache rows below the current position
// and the cross-attention cache are never written by the previous kernel). Per-split math is the
// flash-decoding split of whisper_kernels.cu:108-189; with `counters` set, the last CTA of each
// head to finish merges the splits (the combine of :193-213) so no second launch is needed. The
// arrival counter is an atomic, nothing spins.
struct AttnParams {
  const half* q;
  half* k;
  half* v;
  const half* k_new;
  const half* v_new;
  const int64_t* len_state;
  int max_len;
  float scale;
  float* part_m;
  float* part_l;
  float* part_acc;
  half* out;
  unsigned int* counters;
  // Batched decode: clip z = blockIdx.z reads and writes at these element offsets times z (zero
  // for a single clip); its split partials and arrival counters follow clip z-1's.
  int64_t clip_q, clip_kv, clip_new, clip_out, clip_state;
};

constexpr int kMaxSplits = 128;  // max_len <= 8192 keys

// Merges the splits of one head (the combine of whisper_kernels.cu:193-213, same operation order so
// the result is bit-identical). The split maxima and sums are first staged in shared memory by the
// whole CTA, and the per-split accumulators are loaded 16 at a time, so the merge costs two rounds of
// L2 latency instead of one round per split. Call with all threads of the CTA; threads < 64 write.
__device__ __forceinline__ void combine_head(const float* pm, const float* pl, const float* pa, int splits, half* out,
                                             float* sm, float* sl) {
  for (int s = threadIdx.x; s < splits; s += blockDim.x) {
    sm[s] = __ldcg(pm + s);
    sl[s] = __ldcg(pl + s);
  }
  __syncthreads();
  const int d = threadIdx.x;
  if (d >= kHeadDim) return;
  float m = -INFINITY;
  for (int s = 0; s < splits; ++s) m = fmaxf(m, sm[s]);
  float num = 0.f, den = 0.f;
  for (int s0 = 0; s0 < splits; s0 += 16) {
    float a[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) a[j] = (s0 + j < splits) ? __ldcg(pa + (s0 + j) * kHeadDim + d) : 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int s = s0 + j;
      if (s < splits && sl[s] > 0.f) {
        const float w = __expf(sm[s] - m);
        num = fmaf(a[j], w, num);
        den = fmaf(sl[s], w, den);
      }
    }
  }
  out[d] = __float2half(num / den);
}

// Scratch of one 64-key attention split processed by 64 threads. 16-byte aligned (and so padded)
// because `q` is read as float4.
struct __align__(16) SplitScratch {
  float q[kHeadDim];
  float sc[kSplitKeys];
  float pacc[4][kHeadDim];
  float red[4];
};

// Split scratch plus the staging arrays of the last-CTA combine of attn_split_kernel.
struct __align__(16) UnitScratch {
  SplitScratch s;
  float comb_m[kMaxSplits];
  float comb_l[kMaxSplits];
  int last;
};

// Barrier of the 64 threads that process one split: the whole CTA of the stand-alone kernel (id 0)
// or named barrier `id` (a pair of warps) inside a larger CTA.
__device__ __forceinline__ void unit_sync(int id) {
  if (id == 0)
    __syncthreads();
  else
    asm volatile("bar.sync %0, 64;" ::"r"(id) : "memory");
}

// One 64-key split of one head (whisper_kernels.cu:108-189) on 64 threads, t = 0..63, with the
// query already in U.q (fp32, made visible to the 64 threads by the caller). Thread t scores key t
// over all 64 dims; the 32 pair products fmaf(q0*k0 + q1*k1) are summed in exactly the pairing of
// the reference's warp xor-tree (offsets 16, 8, 4, 2, 1), and the value accumulation keeps the
// reference's per-warp residue classes (keys i = r mod 4, r = 0..3) and their final order, so the
// partial (m, l, acc) is bit-identical to the reference kernel's while the score pass no longer
// serialises a shuffle reduction per key. K rows are read with a per-thread chunk rotation so the
// 16-byte shared loads are bank-conflict free. With kCopies > 1, part_* are this CTA's shared arrays
// and the partial is sent to the same slots of every CTA of the cluster by st.async, counted on
// their mbarrier `xbar` (264 bytes per CTA).
template <int kCopies = 1>
__device__ __forceinline__ void attn_unit64(const half* ks, const half* vs, int n, float scale, int t, SplitScratch& U,
                                            int sync_id, float* part_acc, float* part_m, float* part_l,
                                            uint64_t* xbar = nullptr) {
  const int lane = t & 31, wa = t >> 5;
  float s = -INFINITY;
  if (t < n) {
    const uint4* kr = reinterpret_cast<const uint4*>(ks + t * kHeadDim);
    float pj[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = (j + t) & 7;
      const uint4 kv = kr[c];
      const half2* h2 = reinterpret_cast<const half2*>(&kv);
      const float4 qa = *reinterpret_cast<const float4*>(&U.q[8 * c]);
      const float4 qb = *reinterpret_cast<const float4*>(&U.q[8 * c + 4]);
      const float2 k0 = __half22float2(h2[0]), k1 = __half22float2(h2[1]);
      const float2 k2 = __half22float2(h2[2]), k3 = __half22float2(h2[3]);
      pj[j][0] = fmaf(qa.x, k0.x, qa.y * k0.y);
      pj[j][1] = fmaf(qa.z, k1.x, qa.w * k1.y);
      pj[j][2] = fmaf(qb.x, k2.x, qb.y * k2.y);
      pj[j][3] = fmaf(qb.z, k3.x, qb.w * k3.y);
    }
    // xor-tree pairing: chunk c with c^4, then c^2, then c^1 (rotation keeps the pairs), then
    // within the chunk e with e^2 and e^1
    float a[4][4], b[2][4], cc[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) a[j][e] = pj[j][e] + pj[j + 4][e];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) b[j][e] = a[j][e] + a[j + 2][e];
#pragma unroll
    for (int e = 0; e < 4; ++e) cc[e] = b[0][e] + b[1][e];
    s = ((cc[0] + cc[2]) + (cc[1] + cc[3])) * scale;
  }
  const float wmax = warp_max(s);
  if (lane == 0) U.red[wa] = wmax;
  unit_sync(sync_id);
  const float m = fmaxf(U.red[0], U.red[1]);
  float e = 0.f;
  if (t < n) {
    e = __expf(s - m);
    U.sc[t] = e;
  }
  e = warp_sum(e);
  if (lane == 0) U.red[2 + wa] = e;
  unit_sync(sync_id);
  // value accumulation: warp wa owns residues wa and wa + 2, keys i = wa + 4k in order. The loop
  // has a compile-time trip count so the shared-memory loads are issued ahead of the fma chains.
  float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
#pragma unroll
  for (int k = 0; k < kSplitKeys / 4; ++k) {
    const int i = wa + 4 * k;
    if (i < n) {
      const float2 v0 = __half22float2(reinterpret_cast<const half2*>(vs + i * kHeadDim)[lane]);
      const float p0 = U.sc[i];
      acc0.x = fmaf(p0, v0.x, acc0.x);
      acc0.y = fmaf(p0, v0.y, acc0.y);
    }
    if (i + 2 < n) {
      const float2 v1 = __half22float2(reinterpret_cast<const half2*>(vs + (i + 2) * kHeadDim)[lane]);
      const float p1 = U.sc[i + 2];
      acc1.x = fmaf(p1, v1.x, acc1.x);
      acc1.y = fmaf(p1, v1.y, acc1.y);
    }
  }
  U.pacc[wa][2 * lane] = acc0.x;
  U.pacc[wa][2 * lane + 1] = acc0.y;
  U.pacc[wa + 2][2 * lane] = acc1.x;
  U.pacc[wa + 2][2 * lane + 1] = acc1.y;
  unit_sync(sync_id);
  const float a = ((U.pacc[0][t] + U.pacc[1][t]) + U.pacc[2][t]) + U.pacc[3][t];
  const float l = U.red[2] + U.red[3];
  if (kCopies == 1) {
    part_acc[t] = a;
    if (t == 0) {
      *part_m = m;
      *part_l = l;
    }
  } else {  // the same slots in every CTA of the cluster: this CTA's by plain stores
    const unsigned own = cg::this_cluster().block_rank();
    part_acc[t] = a;
    if (t == 0) {
      *part_m = m;
      *part_l = l;
    }
#pragma unroll
    for (int r = 0; r < kCopies; ++r) {
      if (r == static_cast<int>(own)) continue;
      const uint32_t rb = cluster_map(xbar, r);
      st_async_b32(cluster_map(part_acc + t, r), __float_as_uint(a), rb);
      if (t == 0) {
        st_async_b32(cluster_map(part_m, r), __float_as_uint(m), rb);
        st_async_b32(cluster_map(part_l, r), __float_as_uint(l), rb);
      }
    }
  }
}

// Combine of one head by the 64 threads of a unit (same arithmetic as combine_head).
__device__ __forceinline__ void combine_unit64(UnitScratch& U, int sync_id, int t, const float* pm, const float* pl,
                                               const float* pa, int splits, half* out) {
  for (int s = t; s < splits; s += 64) {
    U.comb_m[s] = __ldcg(pm + s);
    U.comb_l[s] = __ldcg(pl + s);
  }
  unit_sync(sync_id);
  float m = -INFINITY;
  for (int s = 0; s < splits; ++s) m = fmaxf(m, U.comb_m[s]);
  float num = 0.f, den = 0.f;
  for (int s0 = 0; s0 < splits; s0 += 16) {
    float a[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) a[j] = (s0 + j < splits) ? __ldcg(pa + (s0 + j) * kHeadDim + t) : 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int s = s0 + j;
      if (s < splits && U.comb_l[s] > 0.f) {
        const float w = __expf(U.comb_m[s] - m);
        num = fmaf(a[j], w, num);
        den = fmaf(U.comb_l[s], w, den);
      }
    }
  }
  out[t] = __float2half(num / den);
}

// Split-K single-query attention, one 64-key split per 64-thread CTA. The split's K and V rows are
// bulk-copied into shared memory before griddepcontrol.wait (cache rows below the current position
// and the cross-attention cache are never written by the previous kernel). With `counters` set, the
// last CTA of each head to finish merges the splits (atomic arrival counter, nothing spins).
__global__ void __launch_bounds__(64) attn_split_kernel(AttnParams p) {
  __shared__ __align__(128) half ks[kSplitKeys * kHeadDim];
  __shared__ __align__(128) half vs[kSplitKeys * kHeadDim];
  __shared__ __align__(16) UnitScratch U;
  __shared__ __align__(8) uint64_t bar;

  const int head = blockIdx.x;
  const int split = blockIdx.y;
  const int splits = gridDim.y;
  const int z = blockIdx.z;
  if (z > 0) {
    p.q += z * p.clip_q;
    p.k += z * p.clip_kv;
    p.v += z * p.clip_kv;
    if (p.k_new) {
      p.k_new += z * p.clip_new;
      p.v_new += z * p.clip_new;
    }
    if (p.len_state) p.len_state += z * p.clip_state;
    p.out += z * p.clip_out;
    p.part_m += static_cast<size_t>(z) * gridDim.x * splits;
    p.part_l += static_cast<size_t>(z) * gridDim.x * splits;
    p.part_acc += static_cast<size_t>(z) * gridDim.x * splits * kHeadDim;
    if (p.counters) p.counters += z * gridDim.x;
  }
  const int slot = head * splits + split;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;

  int pos = -1;
  int len = p.max_len;
  if (p.len_state) {
    const int64_t raw = p.len_state[0];
    pos = static_cast<int>(raw < 0 ? 0 : (raw >= p.max_len ? p.max_len - 1 : raw));
    if (t == 0 && split == 0 && head == 0 && (raw < 0 || raw >= p.max_len)) flag_error(FW_DEVERR_BAD_INDEX);
    len = pos + 1;
  }
  const int begin = split * kSplitKeys;
  const int n = min(kSplitKeys, len - begin);
  half* kh = p.k + static_cast<size_t>(head) * p.max_len * kHeadDim;
  half* vh = p.v + static_cast<size_t>(head) * p.max_len * kHeadDim;

  if (t == 0) {
    mbar_init(&bar, 1);
    mbar_fence_init();
    if (n > 0) {
      const unsigned bytes = static_cast<unsigned>(n) * kHeadDim * sizeof(half);
      mbar_arrive_expect_tx(&bar, 2 * bytes);
      bulk_g2s(ks, kh + static_cast<size_t>(begin) * kHeadDim, bytes, &bar);
      bulk_g2s(vs, vh + static_cast<size_t>(begin) * kHeadDim, bytes, &bar);
    }
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();

  if (n > 0) {
    if (!mbar_wait(&bar, 0)) flag_error(FW_DEVERR_TIMEOUT);
    if (p.k_new && warp == 0 && pos >= begin && pos < begin + n) {
      const half2 kv = reinterpret_cast<const half2*>(p.k_new + head * kHeadDim)[lane];
      const half2 vv = reinterpret_cast<const half2*>(p.v_new + head * kHeadDim)[lane];
      reinterpret_cast<half2*>(kh + static_cast<size_t>(pos) * kHeadDim)[lane] = kv;  // fused cache write
      reinterpret_cast<half2*>(vh + static_cast<size_t>(pos) * kHeadDim)[lane] = vv;
      reinterpret_cast<half2*>(ks + (pos - begin) * kHeadDim)[lane] = kv;
      reinterpret_cast<half2*>(vs + (pos - begin) * kHeadDim)[lane] = vv;
    }
    if (t < 32) {
      const float2 qf = __half22float2(__ldcg(reinterpret_cast<const half2*>(p.q + head * kHeadDim) + t));
      U.s.q[2 * t] = qf.x;
      U.s.q[2 * t + 1] = qf.y;
    }
    __syncthreads();
    attn_unit64(ks, vs, n, p.scale, t, U.s, 0, p.part_acc + static_cast<size_t>(slot) * kHeadDim, p.part_m + slot,
                p.part_l + slot);
  } else if (t == 0) {
    p.part_m[slot] = -INFINITY;
    p.part_l[slot] = 0.f;
  }

  if (p.counters == nullptr) return;
  // thread 0's acq_rel arrival releases this CTA's partial (ordered before it by the barrier) and, in
  // the last CTA, acquires every other split's
  __syncthreads();
  if (t == 0) U.last = atomic_add_acq_rel(p.counters + head, 1u) == static_cast<unsigned>(splits - 1);
  __syncthreads();
  if (!U.last) return;
  if (t == 0) p.counters[head] = 0u;
  combine_unit64(U, 0, t, p.part_m + head * splits, p.part_l + head * splits,
                 p.part_acc + static_cast<size_t>(head) * splits * kHeadDim, splits, p.out + head * kHeadDim);
}

// Separate combine, used by the reference-compatible entry point.
__global__ void __launch_bounds__(64) attn_combine_kernel(const float* __restrict__ part_m,
                                                          const float* __restrict__ part_l,
                                                          const float* __restrict__ part_acc, half* __restrict__ out,
                                                          int splits) {
  __shared__ float comb_m[kMaxSplits];
  __shared__ float comb_l[kMaxSplits];
  pdl_wait();
  pdl_trigger();
  const int head = blockIdx.x;
  combine_head(part_m + head * splits, part_l + head * splits, part_acc + static_cast<size_t>(head) * splits * kHeadDim,
               splits, out + head * kHeadDim, comb_m, comb_l);
}

// ---------------------------------------------------------------------------------------------
// Attention block of one decoder layer, one thread-block cluster per head. The reference runs
// add_layernorm -> F.linear (q/k/v) -> decode_attention (split + combine) -> F.linear (out_proj)
// -> residual add as five or six launches (custom/model.py:113-116 self, :116-119 cross). Here the
// whole chain is one launch: cluster `head` (kHeadCtas CTAs) computes
//   1. LN(h) and this head's projection rows (q, k, v for self attention; q for cross), split over
//      the cluster's CTAs and broadcast into every CTA's shared memory (DSMEM);
//   2. the 64-key attention splits of this head (self: one per CTA, with the fused cache write;
//      cross: up to kHeadMaxUnits per CTA on 64-thread units), each split's (m, l, acc) broadcast
//      to every CTA;
//   3. the split combine in every CTA (same arithmetic and order as the reference combine);
//   4. this head's slice of the output projection, W_o[:, head] . o_head, for 1280 / kHeadCtas rows
//      per CTA, written as fp32 partials [heads, 1280];
// and leaves the residual update h[r] = fp16(h[r] + fp16(sum over heads, in head order, of the
// partials + b[r])) to the next launch, which forms it itself, each CTA of a cluster for its 160-row
// block, exchanged over DSMEM (`res_part`): the cross block for the self block, fc1
// (ln_gemv_kernel<.., .., true>) for the cross block. So no block needs an arrival counter, a
// last-CTA stage or a write of h that the next launch reads back.
// Weight rows, the K/V splits and the output-projection slice (head-major [heads, 1280, 64]) are
// bulk-copied into shared memory before griddepcontrol.wait. The two exchanges inside the cluster
// (projection rows, split partials) are st.async stores counted on the receiving CTA's mbarrier, so
// a CTA waits only for the bytes it needs, not for every CTA to reach a cluster barrier.
constexpr int kHeads = kHidden / kHeadDim;                // 20
constexpr int kHeadCtas = 8;                              // CTAs per head cluster
constexpr int kHeadMaxUnits = 3;                          // attention splits per CTA (cross: 24 / 8)
constexpr int kOutRows = kHidden / kHeadCtas;             // output-projection rows per CTA (160)
constexpr int kSelfProjRows = 3 * kHeadDim / kHeadCtas;   // q, k, v rows per CTA (24)
constexpr int kCrossProjRows = kHeadDim / kHeadCtas;      // q rows per CTA (8)

struct HeadBlockParams {
  half* h;  // residual stream [1280]: LN input (layer 0's self block writes the embedded row here)
  const half* gamma;
  const half* beta;
  float eps;
  // layer-0 prologue: h is built from the token embedding and learned position instead of read
  const half* embed;
  const half* pos_embed;
  const int64_t* cur;
  const int64_t* prompt;
  int prompt_len;
  int vocab;
  const int64_t* state;  // [position, count]; self attention length = position + 1
  int max_pos;
  bool state_early;  // position may be read before griddepcontrol.wait (no in-flight kernel writes it)
  // projection (self: [3840, 1280] q|k|v rows; cross: [1280, 1280] q rows) and its bias
  const half* w;
  const half* b;
  // attention cache [heads, kv_len, 64]
  half* k;
  half* v;
  int kv_len;
  float scale;
  // output projection, head-major [heads, 1280, 64] (its bias is added by the next launch)
  const half* wo;
  float* part;            // fp32 [heads, 1280] per-head output-projection partials
  half* attn_out;         // optional [heads * 64] attention output (written by rank 0)
  // The residual of the previous attention block (cross block only): the LayerNorm input is
  // h + fp16(sum over heads of res_part + res_bias), formed here.
  const float* res_part;  // [heads, 1280] partials of the previous block, or null
  const half* res_bias;   // [1280] that block's output-projection bias
  half* h_in_out;         // optional [1280]: the formed residual input, written by head 0's CTAs
};

template <bool kSelf>
struct HeadBlockShape {
  static constexpr int kProjRows = kSelf ? kSelfProjRows : kCrossProjRows;
  static constexpr int kUnits = kSelf ? 1 : kHeadMaxUnits;
  static constexpr int kSlots = kHeadCtas * kUnits;
  static constexpr int kProjBytes = kProjRows * kHidden * 2;
  static constexpr int kKvBytes = kUnits * 2 * kSplitKeys * kHeadDim * 2;
  static constexpr int kOutBytes = kOutRows * kHeadDim * 2;
  // projection rows | K/V splits | output-projection slice, all requested before the PDL wait
  static constexpr int kSmem = kProjBytes + kKvBytes + kOutBytes;
};

template <bool kSelf, bool kEmbed>
__global__ void __launch_bounds__(256, 2) head_block_kernel(HeadBlockParams p) {
  using S = HeadBlockShape<kSelf>;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bar_w, bar_kv, bar_o;
  __shared__ __align__(8) uint64_t bar_x, bar_s, bar_h;  // DSMEM exchanges: rows, split partials, residual
  __shared__ float red[16];
  __shared__ __align__(16) half ys[kHidden];
  __shared__ __align__(16) half hs[kHidden];                   // residual-stream input
  __shared__ __align__(16) half qv[S::kProjRows * kHeadCtas];  // this head's q (| k | v)
  __shared__ __align__(16) float os[kHeadDim];                  // this head's attention output
  __shared__ __align__(16) SplitScratch U[S::kUnits];
  __shared__ float sm_m[S::kSlots];
  __shared__ float sm_l[S::kSlots];
  __shared__ __align__(16) float sm_acc[S::kSlots][kHeadDim];
  __shared__ float sm_w[S::kSlots];

  const int rank = blockIdx.x;  // cluster dims (kHeadCtas, 1, 1) over grid (kHeadCtas, heads)
  const int head = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  half* wproj = reinterpret_cast<half*>(smem);
  half* kvs = reinterpret_cast<half*>(smem + S::kProjBytes);
  half* wout = reinterpret_cast<half*>(smem + S::kProjBytes + S::kKvBytes);
  const int splits = (p.kv_len + kSplitKeys - 1) / kSplitKeys;
  half* kh = p.k + static_cast<size_t>(head) * p.kv_len * kHeadDim;
  half* vh = p.v + static_cast<size_t>(head) * p.kv_len * kHeadDim;

  // global projection row of local row j (0 <= j < kProjRows * kHeadCtas)
  auto proj_row = [&](int j) {
    return kSelf ? (j / kHeadDim) * kHidden + head * kHeadDim + (j % kHeadDim) : head * kHeadDim + j;
  };

  // Attention length: self = position + 1 (position read early only when no in-flight kernel
  // writes it), cross = kv_len.
  int pos = 0, len = p.kv_len;
  bool pos_known = !kSelf;
  if (kSelf && p.state_early) {
    pos = static_cast<int>(min(max(p.state[0], int64_t(0)), int64_t(p.max_pos - 1)));
    len = pos + 1;
    pos_known = true;
  }

  // Weights and the cross cache are read once per step: streamed with L2 evict-first.
  const uint64_t stream_policy = policy_evict_first();
  if (tid == 0) {
    mbar_init(&bar_w, 1);
    mbar_init(&bar_kv, 1);
    mbar_init(&bar_o, 1);
    mbar_init(&bar_x, 1);
    mbar_init(&bar_s, 1);
    mbar_init(&bar_h, 1);
    mbar_fence_init();
    mbar_arrive_expect_tx(&bar_x, (kHeadCtas - 1) * S::kProjRows * 2);  // the other CTAs' rows
    if (p.res_part) mbar_arrive_expect_tx(&bar_h, (kHeadCtas - 1) * kOutRows * 2);  // their residual rows
    mbar_arrive_expect_tx(&bar_w, S::kProjBytes);
    for (int r = 0; r < S::kProjRows; ++r)
      bulk_g2s_stream(wproj + r * kHidden, p.w + static_cast<size_t>(proj_row(rank * S::kProjRows + r)) * kHidden,
                      kHidden * 2, &bar_w, stream_policy);
    // K/V rows of this CTA's splits: the keys below the attention length (all of them while the
    // length is not yet known; rows past it are fetched but not used). A unit that attends over
    // n > 0 keys after the wait always had its rows requested here, so it may wait on bar_kv.
    int nkv[S::kUnits];
    unsigned kv_bytes = 0;
    for (int u = 0; u < S::kUnits; ++u) {
      const int begin = (rank * S::kUnits + u) * kSplitKeys;
      nkv[u] = max(0, min(kSplitKeys, (pos_known ? len : p.kv_len) - begin));
      kv_bytes += 2u * static_cast<unsigned>(nkv[u]) * kHeadDim * 2;
    }
    if (kv_bytes) {
      mbar_arrive_expect_tx(&bar_kv, kv_bytes);
      for (int u = 0; u < S::kUnits; ++u) {
        if (nkv[u] == 0) continue;
        const int begin = (rank * S::kUnits + u) * kSplitKeys;
        const unsigned bytes = static_cast<unsigned>(nkv[u]) * kHeadDim * 2;
        if (kSelf) {  // the self cache is small and rewritten every step: default policy
          bulk_g2s(kvs + (2 * u) * kSplitKeys * kHeadDim, kh + static_cast<size_t>(begin) * kHeadDim, bytes, &bar_kv);
          bulk_g2s(kvs + (2 * u + 1) * kSplitKeys * kHeadDim, vh + static_cast<size_t>(begin) * kHeadDim, bytes,
                   &bar_kv);
        } else {
          bulk_g2s_stream(kvs + (2 * u) * kSplitKeys * kHeadDim, kh + static_cast<size_t>(begin) * kHeadDim, bytes,
                          &bar_kv, stream_policy);
          bulk_g2s_stream(kvs + (2 * u + 1) * kSplitKeys * kHeadDim, vh + static_cast<size_t>(begin) * kHeadDim,
                          bytes, &bar_kv, stream_policy);
        }
      }
    }
    mbar_arrive_expect_tx(&bar_o, S::kOutBytes);
    bulk_g2s_stream(wout, p.wo + (static_cast<size_t>(head) * kHidden + rank * kOutRows) * kHeadDim, S::kOutBytes,
                    &bar_o, stream_policy);
  }
  // LayerNorm parameters and biases are weights: loaded before the wait, into registers
  constexpr int kRowsPerWarp = (S::kProjRows + 7) / 8;
  float g[5], be[5], pbias[kRowsPerWarp];
#pragma unroll
  for (int i = 0; i < 5; ++i) {
    g[i] = __half2float(p.gamma[tid + i * 256]);
    be[i] = __half2float(p.beta[tid + i * 256]);
  }
#pragma unroll
  for (int i = 0; i < kRowsPerWarp; ++i) {
    const int r = warp + 8 * i;
    pbias[i] = (p.b && r < S::kProjRows) ? __half2float(p.b[proj_row(rank * S::kProjRows + r)]) : 0.f;
  }
  __syncthreads();
  cluster_arrive_relaxed();  // completed by the wait before the first DSMEM store: all CTAs are running
  pdl_wait();
  if (kSelf) pdl_trigger();  // (the cross block releases fc1 later, see below)

  // ---- 1. LayerNorm prologue and this CTA's projection rows ----
  if (kEmbed || (kSelf && !p.state_early)) {
    const int64_t raw = p.state[0];
    if (raw < 0 || raw >= p.max_pos) {
      if (tid == 0 && rank == 0 && head == 0) flag_error(FW_DEVERR_BAD_INDEX);
    }
    pos = static_cast<int>(min(max(raw, int64_t(0)), int64_t(p.max_pos - 1)));
    len = pos + 1;
  }
  if (tid == 0) {  // partials of the other CTAs' splits: 66 floats each, (m, l) alone for an empty split
    unsigned sb = 0;
    for (int sp = 0; sp < splits; ++sp)
      if (sp / S::kUnits != rank) sb += (len - sp * kSplitKeys > 0) ? (kHeadDim + 2) * 4u : 8u;
    mbar_arrive_expect_tx(&bar_s, sb);
  }
  float v[5];
  if (kEmbed) {
    int64_t tok = (pos < p.prompt_len) ? p.prompt[pos] : p.cur[0];
    if (tok < 0 || tok >= p.vocab) {
      if (tid == 0 && rank == 0 && head == 0) flag_error(FW_DEVERR_BAD_INDEX);
      tok = tok < 0 ? 0 : p.vocab - 1;
    }
    const half* er = p.embed + static_cast<size_t>(tok) * kHidden;
    const half* pr = p.pos_embed + static_cast<size_t>(pos) * kHidden;
#pragma unroll
    for (int i = 0; i < 5; ++i) v[i] = round_half(__half2float(er[tid + i * 256]) + __half2float(pr[tid + i * 256]));
  } else if (p.res_part) {
    // this CTA's 160 rows of h_in = h + fp16(sum over heads, in order, of the previous block's partials
    // + its bias) — the previous block's last-CTA arithmetic — then the rows to the cluster's other CTAs
    cluster_wait();  // every CTA of the cluster is running (its mbarriers initialised)
    if (tid < kOutRows) {
      const int e = rank * kOutRows + tid;
      float pv[kHeads];
#pragma unroll
      for (int hh = 0; hh < kHeads; ++hh) pv[hh] = __ldcg(p.res_part + static_cast<size_t>(hh) * kHidden + e);
      const float h0 = __half2float(p.h[e]), rb = __half2float(p.res_bias[e]);
      float acc = 0.f;
#pragma unroll
      for (int hh = 0; hh < kHeads; ++hh) acc += pv[hh];
      const half hv = __float2half(h0 + round_half(acc + rb));
      hs[e] = hv;
      if (p.h_in_out && head == 0) p.h_in_out[e] = hv;
    }
    __syncthreads();
    constexpr int kChunks = kOutRows * 2 / 16;  // 16-byte pieces of the 160-row block
    if (tid < (kHeadCtas - 1) * kChunks) {
      const int dst = tid / kChunks + (tid / kChunks >= rank ? 1 : 0), c = tid % kChunks;
      const uint4 val = reinterpret_cast<const uint4*>(hs + rank * kOutRows)[c];
      st_async_v4(cluster_map(hs + rank * kOutRows, dst) + 16 * c, val, cluster_map(&bar_h, dst));
    }
    if (!mbar_wait_cluster(&bar_h, 0)) flag_error(FW_DEVERR_TIMEOUT);
#pragma unroll
    for (int i = 0; i < 5; ++i) v[i] = __half2float(hs[tid + i * 256]);
  } else {
#pragma unroll
    for (int i = 0; i < 5; ++i) v[i] = __half2float(p.h[tid + i * 256]);
  }
#pragma unroll
  for (int i = 0; i < 5; ++i) hs[tid + i * 256] = __float2half(v[i]);  // exact: v holds fp16 values
  float mean, inv;
  ln1280_stats(v, red, p.eps, mean, inv);
#pragma unroll
  for (int i = 0; i < 5; ++i) ys[tid + i * 256] = __float2half(ln_apply(v[i], mean, inv, g[i], be[i]));
  __syncthreads();
  {
    float xf[40];
    load_x40(ys, xf);
    if (!mbar_wait(&bar_w, 0)) flag_error(FW_DEVERR_TIMEOUT);
    if (!p.res_part) cluster_wait();  // (already waited for in the residual exchange)
    static_assert(S::kProjRows % 8 == 0, "projection rows must fill the 8 warps evenly");
    float acc[kRowsPerWarp];
    dot1280_rows<kRowsPerWarp>(wproj + warp * kHidden, 8 * kHidden, xf, acc);
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < kRowsPerWarp; ++i) qv[rank * S::kProjRows + warp + 8 * i] = __float2half(acc[i] + pbias[i]);
    }
  }
  __syncthreads();
  if (tid < kHeadCtas && tid != rank) {  // this CTA's rows into the same place of every other CTA
    const uint4* src = reinterpret_cast<const uint4*>(qv + rank * S::kProjRows);
    const uint32_t dst = cluster_map(qv + rank * S::kProjRows, tid), rb = cluster_map(&bar_x, tid);
#pragma unroll
    for (int c = 0; c < S::kProjRows * 2 / 16; ++c) st_async_v4(dst + 16 * c, src[c], rb);
  }
  if (!mbar_wait_cluster(&bar_x, 0)) flag_error(FW_DEVERR_TIMEOUT);  // q (| k | v) of this head complete
  // The cross block releases fc1 only now: fc1's weight prefetch (a burst of bulk copies) would
  // otherwise queue in front of this kernel's loads, and this kernel runs long enough after this point
  // for that prefetch to complete. (The self block releases the cross block right after its wait:
  // measured 0.4 us per token faster; the cross block doing the same was 1.7 us slower.)
  if (!kSelf) pdl_trigger();

  // ---- 2. attention splits ----
  {
    const int u = tid >> 6, t = tid & 63;
    const int split = rank * S::kUnits + u;
    if (u < S::kUnits && split < splits) {
      const int begin = split * kSplitKeys;
      const int n = min(kSplitKeys, len - begin);
      half* ks = kvs + (2 * u) * kSplitKeys * kHeadDim;
      half* vs = kvs + (2 * u + 1) * kSplitKeys * kHeadDim;
      if (n > 0) {
        if (!mbar_wait(&bar_kv, 0)) flag_error(FW_DEVERR_TIMEOUT);
        if constexpr (kSelf) {
          if (t < 32 && pos >= begin && pos < begin + n) {  // fused cache write of the new key/value
            const half2 kn = reinterpret_cast<const half2*>(qv + kHeadDim)[t];
            const half2 vn = reinterpret_cast<const half2*>(qv + 2 * kHeadDim)[t];
            reinterpret_cast<half2*>(kh + static_cast<size_t>(pos) * kHeadDim)[t] = kn;
            reinterpret_cast<half2*>(vh + static_cast<size_t>(pos) * kHeadDim)[t] = vn;
            reinterpret_cast<half2*>(ks + (pos - begin) * kHeadDim)[t] = kn;
            reinterpret_cast<half2*>(vs + (pos - begin) * kHeadDim)[t] = vn;
          }
        }
        if (t < 32) {
          const float2 qf = __half22float2(reinterpret_cast<const half2*>(qv)[t]);
          U[u].q[2 * t] = qf.x;
          U[u].q[2 * t + 1] = qf.y;
        }
        unit_sync(1 + u);
        attn_unit64<kHeadCtas>(ks, vs, n, p.scale, t, U[u], 1 + u, &sm_acc[split][0], &sm_m[split], &sm_l[split],
                               &bar_s);
      } else if (t == 0) {
        sm_m[split] = -INFINITY;
        sm_l[split] = 0.f;
#pragma unroll
        for (int r = 0; r < kHeadCtas; ++r) {
          if (r == rank) continue;
          const uint32_t rb = cluster_map(&bar_s, r);
          st_async_b32(cluster_map(&sm_m[split], r), __float_as_uint(-INFINITY), rb);
          st_async_b32(cluster_map(&sm_l[split], r), __float_as_uint(0.f), rb);
        }
      }
    }
  }
  if (!mbar_wait_cluster(&bar_s, 0)) flag_error(FW_DEVERR_TIMEOUT);  // every split's partial received
  // No CTA exits before all have received their partials (the wait at each exit below), so no st.async
  // targets a CTA that has exited.
  cluster_arrive_relaxed();
  __syncthreads();  // this CTA's own partials (plain stores) visible to all its threads

  // ---- 3. split combine (whisper_kernels.cu:193-213 order), in every CTA: the split weights
  // exp(m_s - m) are computed one per thread, then the sums run in split order ----
  if (tid < splits) {
    float m = -INFINITY;
#pragma unroll
    for (int s = 0; s < S::kSlots; ++s)
      if (s < splits) m = fmaxf(m, sm_m[s]);
    sm_w[tid] = sm_l[tid] > 0.f ? __expf(sm_m[tid] - m) : 0.f;
  }
  __syncthreads();
  if (tid < kHeadDim) {
    float num = 0.f, den = 0.f;
#pragma unroll
    for (int s = 0; s < S::kSlots; ++s) {
      if (s < splits && sm_l[s] > 0.f) {
        const float w = sm_w[s];
        num = fmaf(sm_acc[s][tid], w, num);
        den = fmaf(sm_l[s], w, den);
      }
    }
    const half o = __float2half(num / den);
    os[tid] = __half2float(o);
    if (p.attn_out && rank == 0) p.attn_out[head * kHeadDim + tid] = o;
  }
  __syncthreads();

  // ---- 4. this head's output-projection partial for rows rank*160 .. +159 ----
  const int row0 = rank * kOutRows;
  if (!mbar_wait(&bar_o, 0)) flag_error(FW_DEVERR_TIMEOUT);
  if (tid < kOutRows) {
    const uint4* wr = reinterpret_cast<const uint4*>(wout + tid * kHeadDim);
    const float4* o4 = reinterpret_cast<const float4*>(os);
    float acc2[2] = {0.f, 0.f};  // two chains: even and odd steps of the rotated chunk order
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = (j + tid) & 7;  // rotation keeps the 16-byte shared loads conflict-free
      const uint4 wv = wr[c];
      const float4 oa = o4[2 * c], ob = o4[2 * c + 1];
      const half2* w2 = reinterpret_cast<const half2*>(&wv);
      const float2 f0 = __half22float2(w2[0]), f1 = __half22float2(w2[1]);
      const float2 f2 = __half22float2(w2[2]), f3 = __half22float2(w2[3]);
      float& a = acc2[j & 1];
      a = fmaf(f0.x, oa.x, a);
      a = fmaf(f0.y, oa.y, a);
      a = fmaf(f1.x, oa.z, a);
      a = fmaf(f1.y, oa.w, a);
      a = fmaf(f2.x, ob.x, a);
      a = fmaf(f2.y, ob.y, a);
      a = fmaf(f3.x, ob.z, a);
      a = fmaf(f3.y, ob.w, a);
    }
    __stcg(p.part + static_cast<size_t>(head) * kHidden + row0 + tid, acc2[0] + acc2[1]);
  }

  // ---- 5. the residual is formed by the next launch; layer 0 built h from the embedding, which the
  // next block reads from p.h ----
  if (kEmbed && head == 0 && tid < kOutRows) p.h[row0 + tid] = hs[row0 + tid];
  cluster_wait();  // no CTA exits while a peer may still send it exchange bytes
}

// ---------------------------------------------------------------------------------------------
// LM head: fused (optional final LayerNorm) + GEMV over the vocab + argmax (+ optional finalize).
// One CTA per SM owns a contiguous range of vocab rows; each of its 8 warps streams its own
// contiguous share through a private ring of kLmSlots shared-memory slots (kLmSlotRows rows each,
// 160 KB per CTA)
// fed by bulk async copies issued by the warp's lane 0. Warps never wait for one another inside the
// loop, so a slot is refilled as soon as its warp has consumed it and the bytes in flight stay high
// while other warps compute; two rows per slot are dotted together to overlap their latency. The
// first slots are requested before griddepcontrol.wait.
constexpr int kLmSlots = 4;
constexpr int kLmSlotRows = 2;
constexpr int kLmSlotBytes = kLmSlotRows * kHidden * 2;
constexpr int kLmSmem = 8 * kLmSlots * kLmSlotBytes;
constexpr int kLmMaxRowsPerCta = 512;  // vocab <= 512 * SMs

struct LmParams {
  const half* h;
  const half* gamma;
  const half* beta;
  float eps;
  const half* w;
  const int8_t* wq;   // lm_head_q_kernel: int8 rows and per-row {scale, a, c2, 0} (fw_lm_quantize)
  const float4* rp;
  int vocab;
  int rows_per_cta;
  const bool* mask;
  const bool* first_mask;
  unsigned long long* best;
  // finalize
  unsigned int* counter;
  int64_t* tokens;
  int64_t n_tokens;
  int64_t* state;
  int64_t* cur;
  int max_pos;
  int prompt_len;
  half* y_out;  // optional [1280]: CTA 0 writes the (LayerNorm) input row it dotted (fw_decoder_step_trace)
  // batched decode (lm_head_q_kernel<.., .., kClips > 1>): clip count and row stride of tokens
  int clips;
  int64_t tokens_stride;
};

// Token bookkeeping shared by argmax_finalize and the fused LM-head tail.
// Reference semantics: whisper_kernels.cu:90-100, with the prompt handling of
// custom/model.py:197-207 moved onto the device (prompt predictions are discarded).
__device__ __forceinline__ void finalize_token(unsigned long long b, int64_t* tokens, int64_t n_tokens, int64_t* state,
                                               int64_t* cur, int max_pos, int prompt_len) {
  const int64_t tok = static_cast<int64_t>(0xFFFFFFFFu - static_cast<unsigned int>(b & 0xFFFFFFFFull));
  const int64_t pos = state[0];
  if (prompt_len > 0 && pos < prompt_len - 1) {
    state[0] = pos + 1 < max_pos ? pos + 1 : max_pos - 1;
    *cur = tok;
    return;
  }
  const int64_t n = state[1];
  if (n < max_pos && n < n_tokens) tokens[n] = tok;
  state[1] = n < max_pos ? n + 1 : n;
  state[0] = pos + 1 < max_pos ? pos + 1 : max_pos - 1;
  *cur = tok;
}

template <bool kLN, bool kFinalize>
__global__ void __launch_bounds__(256) lm_head_kernel(LmParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[8][kLmSlots];
  __shared__ float red[16];
  __shared__ __align__(16) half ys[kHidden];
  __shared__ unsigned long long warp_best[8];
  __shared__ uint8_t msk[2][kLmMaxRowsPerCta];  // suppress flags of this CTA's rows: base, first step
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r0 = blockIdx.x * p.rows_per_cta;
  const int r1 = min(p.vocab, r0 + p.rows_per_cta);
  const int nrows = max(0, r1 - r0);
  // this warp's rows
  const int per_warp = (nrows + 7) / 8;
  const int w0 = r0 + warp * per_warp;
  const int wn = max(0, min(r1, w0 + per_warp) - w0);
  const int nst = (wn + kLmSlotRows - 1) / kLmSlotRows;
  uint8_t* ring = smem + warp * kLmSlots * kLmSlotBytes;
  const uint64_t policy = policy_evict_first();
  auto issue = [&](int st, int slot) {
    const int rows = min(kLmSlotRows, wn - st * kLmSlotRows);
    const unsigned bytes = static_cast<unsigned>(rows) * kHidden * 2;
    mbar_arrive_expect_tx(&full[warp][slot], bytes);
    bulk_g2s_stream(ring + slot * kLmSlotBytes, p.w + static_cast<size_t>(w0 + st * kLmSlotRows) * kHidden, bytes,
                    &full[warp][slot], policy);
  };

  if (lane == 0) {
    for (int s = 0; s < kLmSlots; ++s) mbar_init(&full[warp][s], 1);
    mbar_fence_init();
    for (int s = 0; s < kLmSlots && s < nst; ++s) issue(s, s);
  }
  // The suppress masks are constant: staged before the wait so the row loop reads shared memory.
  for (int i = threadIdx.x; i < nrows; i += 256) {
    msk[0][i] = p.mask ? static_cast<uint8_t>(p.mask[r0 + i]) : 0;
    msk[1][i] = p.first_mask ? static_cast<uint8_t>(p.first_mask[r0 + i]) : 0;
  }
  float g[5], be[5];  // final LayerNorm parameters, loaded before the wait
  if (kLN) {
#pragma unroll
    for (int i = 0; i < 5; ++i) {
      g[i] = __half2float(p.gamma[threadIdx.x + i * 256]);
      be[i] = __half2float(p.beta[threadIdx.x + i * 256]);
    }
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();

  if (kLN) {
    float v[5];
#pragma unroll
    for (int i = 0; i < 5; ++i) v[i] = __half2float(p.h[threadIdx.x + i * 256]);
    float mean, inv;
    ln1280_stats(v, red, p.eps, mean, inv);
#pragma unroll
    for (int i = 0; i < 5; ++i) ys[threadIdx.x + i * 256] = __float2half(ln_apply(v[i], mean, inv, g[i], be[i]));
  } else {
#pragma unroll
    for (int i = 0; i < 5; ++i) ys[threadIdx.x + i * 256] = p.h[threadIdx.x + i * 256];
  }
  __syncthreads();
  if (p.y_out && blockIdx.x == 0) {
#pragma unroll
    for (int i = 0; i < 5; ++i) p.y_out[threadIdx.x + i * 256] = ys[threadIdx.x + i * 256];
  }
  float xf[40];
  load_x40(ys, xf);

  const uint8_t* mask = msk[0];
  if (kFinalize && p.first_mask && p.prompt_len > 0 && p.state[0] == p.prompt_len - 1) mask = msk[1];

  unsigned long long mine = 0;
  auto take = [&](float acc, int row) {  // logits are fp16 in the reference (whisper_kernels.cu:70-71)
    if (!mask[row - r0]) {
      const unsigned long long key = pack_score(round_half(acc), row);
      mine = key > mine ? key : mine;
    }
  };
  for (int s = 0; s < nst; ++s) {
    const int slot = s % kLmSlots;
    if (!mbar_wait(&full[warp][slot], (s / kLmSlots) & 1)) flag_error(FW_DEVERR_TIMEOUT);
    const int row = w0 + s * kLmSlotRows;
    const half* base = reinterpret_cast<const half*>(ring + slot * kLmSlotBytes);
    if (row + kLmSlotRows <= w0 + wn) {
      float acc[kLmSlotRows];
      dot1280_rows<kLmSlotRows>(base, kHidden, xf, acc);
      if (lane == 0) {
#pragma unroll
        for (int i = 0; i < kLmSlotRows; ++i) take(acc[i], row + i);
      }
    } else {
      for (int i = 0; row + i < w0 + wn; ++i) {
        float acc[1];
        dot1280_rows<1>(base + i * kHidden, kHidden, xf, acc);
        if (lane == 0) take(acc[0], row + i);
      }
    }
    __syncwarp();  // every lane is done reading the slot before it is refilled
    if (lane == 0 && s + kLmSlots < nst) issue(s + kLmSlots, slot);
  }
  if (lane == 0) warp_best[warp] = mine;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long m = 0;
    for (int i = 0; i < 8; ++i) m = warp_best[i] > m ? warp_best[i] : m;
    if (m) atomicMax(p.best, m);
    if (kFinalize) {  // the acq_rel arrival releases this CTA's maximum and, in the last CTA, acquires all
      if (atomic_add_acq_rel(p.counter, 1u) == gridDim.x - 1) {
        const unsigned long long b = atomicExch(p.best, 0ull);
        finalize_token(b, p.tokens, p.n_tokens, p.state, p.cur, p.max_pos, p.prompt_len);
        *p.counter = 0u;
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------
// Pruned LM head: the same argmax as lm_head_kernel, reading half the bytes.
//
// fw_lm_quantize stores each vocab row w_r as int8 q_r with a per-row scale s_r (s_r = max|w_r| /
// 127) and two per-row error terms, computed exactly in fp64 and rounded up to fp32:
//   a_r  = max_i |w_ri - s_r q_ri| + 1e-5 max_i |w_ri|
//   c2_r = 0.51 s_r sum_i |q_ri|
// The kernel quantises the LayerNorm output x to 14-bit integers xq (scale sx = max|x| / 8191, so
// |x_i - sx xq_i| <= 0.51 sx), splits them as xq = 128 x_hi + x_lo with x_hi in [-64, 64] and x_lo in
// [-64, 63] (both int8), streams q, and forms the exact integer S_r = sum_i xq_i q_ri = 128 v0 + v1
// from the two int32 columns v0 = sum_i q_ri x_hi_i and v1 = sum_i q_ri x_lo_i of a tcgen05.mma
// kind::i8 against B = [x_hi; x_lo]. The int32 accumulators cannot overflow: |v0|, |v1| <= 1280 * 127
// * 64 < 2^31, and |S_r| <= 1280 * 127 * 8191 < 2^31. approx_r = s_r sx S_r then satisfies |dot_r - approx_r| <= B_r with
//   B_r = (|x|_1 a_r + sx c2_r + 4e-7 |approx_r|) (1 + 1e-5),
// where dot_r is the fp32 value the exact kernel computes (its own rounding error is at most
// 45 * 2^-24 |x|_1 max|w_r|, inside the 1e-5 term; the other terms bound the two quantisations
// and the fp32 rounding of approx_r). With L_r = approx_r - B_r, U_r = approx_r + B_r and
// T = max over this CTA's unsuppressed rows of L_r, a row with U_r < T - m, m = 2^-9 (|T| + 2 max
// B) + 2^-23, has fp16(dot_r) strictly below fp16(dot) of the row that set T (the margin exceeds
// the fp16 spacing at those magnitudes), so it can neither win nor tie. The CTA recomputes the
// remaining rows exactly with dot1280 (the arithmetic of lm_head_kernel, bit for bit) and takes
// the packed-key maximum of those; the global argmax row is always among its CTA's survivors, so
// the result equals lm_head_kernel's. If T is not finite or |T| >= 32768 (fp16 overflow makes
// distant values tie at infinity) every unsuppressed row of the CTA is recomputed.
constexpr int kQStagesMax = 8;                          // TMA ring depth (16 KB stages), batched head
constexpr int kQTileRows = 128;                         // MMA M: vocab rows per accumulator tile
constexpr int kQBoxRows = 32;                           // rows per TMA box
constexpr int kQChunk = 128;                            // K bytes per stage (one 128-byte swizzle row)
constexpr int kQChunks = kHidden / kQChunk;             // 10 stages per tile
constexpr int kQStageBytes = kQTileRows * kQChunk;      // 16 KB
constexpr float kXqMax = 8191.f;

__device__ __forceinline__ void tc_mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// kind::i8 instruction descriptor: D s32 (bits 4-5 = 2), A and B signed int8 (bits 7-9, 10-12 = 1),
// both K-major, N >> 3 at bits 17-22, M >> 4 at bits 24-28.
__host__ __device__ constexpr uint32_t make_idesc_s8(int m, int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}
__device__ __forceinline__ void tc_ld2(uint32_t taddr, uint32_t& a, uint32_t& b) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];" : "=r"(a), "=r"(b) : "r"(taddr) : "memory");
}
__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}

// Exact fp32 dot of kRows fp16 rows at arbitrary addresses with x: per row the arithmetic of
// dot1280_rows (lane order, fma chain, butterfly), so the results are bit-identical to it.
template <int kRows>
__device__ __forceinline__ void dot1280_ptrs(const half* const (&rows)[kRows], const float (&xf)[40],
                                             float (&out)[kRows]) {
  const int lane = threadIdx.x & 31;
  float acc[kRows];
#pragma unroll
  for (int r = 0; r < kRows; ++r) acc[r] = 0.f;
  uint4 wv[kRows][5];
#pragma unroll
  for (int c = 0; c < 5; ++c)
#pragma unroll
    for (int r = 0; r < kRows; ++r) wv[r][c] = __ldg(reinterpret_cast<const uint4*>(rows[r]) + lane + 32 * c);
#pragma unroll
  for (int c = 0; c < 5; ++c) {
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      const half2* p = reinterpret_cast<const half2*>(&wv[r][c]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(p[k]);
        acc[r] = fmaf(f.x, xf[c * 8 + 2 * k], acc[r]);
        acc[r] = fmaf(f.y, xf[c * 8 + 2 * k + 1], acc[r]);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int r = 0; r < kRows; ++r) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
#pragma unroll
  for (int r = 0; r < kRows; ++r) out[r] = acc[r];
}

// Shape of lm_head_q_kernel for up to kClips clips: the B operand holds (x_hi, x_lo) of every clip
// in rows 2c, 2c + 1 (MMA N = 8 for one clip, 16 for up to eight), the accumulator of each tile is
// N TMEM columns (two buffers), and the per-clip arrays live in dynamic shared memory after the
// stage ring.
template <int kClips>
struct LmqShape {
  // The batch-1 head keeps 6 stages so that a CTA (122 KB of shared memory) fits on an SM beside one
  // of the preceding fc2 launch (103 KB): it then starts, and requests its first stages, while fc2
  // runs instead of after it.
  static constexpr int kStages = kClips == 1 ? 6 : kQStagesMax;
  static constexpr int kN = 2 * kClips <= 8 ? 8 : 16;
  static constexpr int kXBytes = kQChunks * kN * kQChunk;
  static constexpr int kYsOff = kStages * kQStageBytes + kXBytes;
  static constexpr int kUbOff = kYsOff + kClips * kHidden * 2;
  static constexpr int kCandOff = kUbOff + kClips * kLmMaxRowsPerCta * 4;
  static constexpr int kSmem = kCandOff + kClips * kLmMaxRowsPerCta * 2 + 1024;
  static constexpr uint32_t kTmemCols = 2 * kN <= 32 ? 32 : 64;
};

// Warp roles: warp 0 streams the CTA's int8 rows (32-row x 128-byte TMA boxes, 128B swizzle) through
// a kStages ring, the first stages requested before the PDL wait; warp 1 owns TMEM and issues
// tcgen05.mma kind::i8 (M = 128 rows, N = 8 or 16, K = 32) of each tile against the B operand
// [x_hi; x_lo] of every clip (xq = 128 x_hi + x_lo, both int8) into one of two TMEM accumulators;
// warps 2-5 read each row's two int32 sums per clip (tcgen05.ld, TMEM lane = row) and form approx_r
// and B_r; all eight warps then select and rescore the surviving rows of each clip. kClips > 1 is the
// batched decode step (p.clips <= kClips clips; clip c's LayerNorm input at p.h + 1280 c, its key at
// p.best[c], its bookkeeping at p.state + 2c, p.cur + c and p.tokens + c * p.tokens_stride).
template <bool kLN, bool kFinalize, int kClips>
__global__ void __launch_bounds__(256, 1) lm_head_q_kernel(const __grid_constant__ CUtensorMap tmW, LmParams p) {
  using S = LmqShape<kClips>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full[S::kStages];
  __shared__ __align__(8) uint64_t empty[S::kStages];
  __shared__ __align__(8) uint64_t acc_full[2];
  __shared__ __align__(8) uint64_t acc_empty[2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ float red[16];
  __shared__ float ln_g[kClips > 1 ? kHidden : 1], ln_b[kClips > 1 ? kHidden : 1];  // final LN (several clips)
  __shared__ __align__(16) float4 rps[kLmMaxRowsPerCta];
  __shared__ uint8_t msk[2][kLmMaxRowsPerCta];
  __shared__ float warp_l[kClips][8], warp_b[kClips][8], xstat[kClips][2][8];
  __shared__ unsigned long long warp_best[kClips][8];
  __shared__ int ncand[kClips];
  __shared__ unsigned s_lo_max[kClips];  // running max of the lower bounds (order-preserving bits)
  __shared__ unsigned s_b_max[kClips];   // several clips: max of the bounds (order-preserving bits)
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* stages = smem_raw + (base - raw);
  uint8_t* xb = stages + S::kStages * kQStageBytes;
  half* ys = reinterpret_cast<half*>(stages + S::kYsOff);                // [kClips][1280]
  float* ub = reinterpret_cast<float*>(stages + S::kUbOff);              // [kClips][kLmMaxRowsPerCta]
  unsigned short* cand = reinterpret_cast<unsigned short*>(stages + S::kCandOff);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int C = kClips == 1 ? 1 : p.clips;
  const int r0 = blockIdx.x * p.rows_per_cta;
  const int r1 = min(p.vocab, r0 + p.rows_per_cta);
  const int nrows = max(0, r1 - r0);
  const int n_tiles = (nrows + kQTileRows - 1) / kQTileRows;
  const int total = n_tiles * kQChunks;
  auto issue = [&](int it, uint64_t policy) {
    const int t = it / kQChunks, c = it - t * kQChunks, s = it % S::kStages;
    const int boxes = (min(kQTileRows, nrows - t * kQTileRows) + kQBoxRows - 1) / kQBoxRows;
    mbar_arrive_expect_tx(&full[s], static_cast<unsigned>(boxes * kQBoxRows * kQChunk));
    for (int b = 0; b < boxes; ++b)
      tma_load_2d_hint(stages + s * kQStageBytes + b * kQBoxRows * kQChunk, &tmW, &full[s], c * kQChunk,
                       r0 + t * kQTileRows + b * kQBoxRows, policy);
  };

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < S::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_fence_init();
    tma_prefetch_desc(&tmW);
    const uint64_t policy = policy_evict_first();
    for (int it = 0; it < S::kStages && it < total; ++it) issue(it, policy);  // weights: before the wait
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_sh, S::kTmemCols);
    tmem_relinquish();
  }
  // Constant per-row data (suppress flags, scales and bounds) and the zero rows of B.
  for (int i = threadIdx.x; i < nrows; i += 256) {
    msk[0][i] = p.mask ? static_cast<uint8_t>(p.mask[r0 + i]) : 0;
    msk[1][i] = p.first_mask ? static_cast<uint8_t>(p.first_mask[r0 + i]) : 0;
    rps[i] = p.rp[r0 + i];
  }
  for (int i = threadIdx.x; i < S::kXBytes / 16; i += 256) reinterpret_cast<uint4*>(xb)[i] = make_uint4(0, 0, 0, 0);
  if (threadIdx.x < kClips) {
    ncand[threadIdx.x] = 0;
    s_lo_max[threadIdx.x] = float_to_ordered(-INFINITY);
    s_b_max[threadIdx.x] = float_to_ordered(0.f);
  }
  float g[5], be[5];
  if (kLN) {
#pragma unroll
    for (int i = 0; i < 5; ++i) {
      g[i] = __half2float(p.gamma[threadIdx.x + i * 256]);
      be[i] = __half2float(p.beta[threadIdx.x + i * 256]);
      if (kClips > 1) {
        ln_g[threadIdx.x + i * 256] = g[i];
        ln_b[threadIdx.x + i * 256] = be[i];
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  pdl_wait();
  pdl_trigger();

  // LayerNorm of each clip's row, its max|x| and |x|_1, and the B operand rows 2c (x_hi) and 2c + 1
  // (x_lo) of xq = rint(x / sx). 16-byte unit j of row n of an 8-row 128B-swizzled atom is stored at
  // unit j ^ (n % 8); rows 8..15 form the second atom of the K chunk.
  auto put_b = [&](int n, int k, int val) {
    const int ch = k >> 7, kk = k & 127;
    xb[ch * S::kN * kQChunk + (n >> 3) * 1024 + (n & 7) * kQChunk + ((((kk >> 4) ^ (n & 7)) & 7) << 4) + (kk & 15)] =
        static_cast<uint8_t>(static_cast<int8_t>(val));
  };
  auto put_xq = [&](int c, int k, float x, float xinv) {
    const int xq = max(-8191, min(8191, __float2int_rn(x * xinv)));
    const int xh = (xq + 64) >> 7;  // floor((xq + 64) / 128), in [-64, 64]
    put_b(2 * c, k, xh);
    put_b(2 * c + 1, k, xq - (xh << 7));  // in [-64, 63]
  };
  float sx[kClips], nx1[kClips];
  if constexpr (kClips == 1) {
    // all 256 threads on the one row, ln1280_stats order
    float xv[5];
    if (kLN) {
#pragma unroll
      for (int i = 0; i < 5; ++i) xv[i] = __half2float(p.h[threadIdx.x + i * 256]);
      float mean, inv;
      ln1280_stats(xv, red, p.eps, mean, inv);
#pragma unroll
      for (int i = 0; i < 5; ++i) {
        const half y = __float2half(ln_apply(xv[i], mean, inv, g[i], be[i]));
        ys[threadIdx.x + i * 256] = y;
        xv[i] = __half2float(y);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 5; ++i) {
        const half y = p.h[threadIdx.x + i * 256];
        ys[threadIdx.x + i * 256] = y;
        xv[i] = __half2float(y);
      }
    }
    if (p.y_out && blockIdx.x == 0) {
#pragma unroll
      for (int i = 0; i < 5; ++i) p.y_out[threadIdx.x + i * 256] = __float2half(xv[i]);
    }
    float mx = 0.f, sm = 0.f;
#pragma unroll
    for (int i = 0; i < 5; ++i) {
      mx = fmaxf(mx, fabsf(xv[i]));
      sm += fabsf(xv[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      sm += __shfl_xor_sync(0xffffffffu, sm, o);
    }
    if (lane == 0) {
      xstat[0][0][warp] = mx;
      xstat[0][1][warp] = sm;
    }
    __syncthreads();
    float xmax = 0.f, n1 = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      xmax = fmaxf(xmax, xstat[0][0][i]);
      n1 += xstat[0][1][i];
    }
    nx1[0] = n1 * 1.0001f;  // covers the fp32 rounding of the sum
    sx[0] = xmax > 0.f ? xmax / kXqMax : 0.f;
    const float xinv = xmax > 0.f ? kXqMax / xmax : 0.f;
#pragma unroll
    for (int i = 0; i < 5; ++i) put_xq(0, threadIdx.x + i * 256, xv[i], xinv);
  } else {
    // Warp w normalises clip w by itself. Its 32 lanes stand in for the 256 threads of ln1280_stats
    // one warp-row at a time (virtual warp j = threads 32j .. 32j + 31), so the per-thread sums, the
    // xor-trees and the ordered sum of the eight warp partials are exactly ln1280_stats'. The code is
    // one short loop per clip rather than eight unrolled copies. (|x|_1 only scales a bound, which
    // the 1.0001 factor keeps rigorous in any summation order.)
    const int c = warp;
    if (c < C) {
      const half* hc = p.h + c * kHidden;
      half* yc = ys + c * kHidden;
      float v[8][5];
      float part[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float sum = 0.f;
#pragma unroll
        for (int i = 0; i < 5; ++i) {
          v[j][i] = __half2float(hc[32 * j + lane + 256 * i]);
          sum += v[j][i];
        }
        part[j] = warp_sum(sum);
      }
      if (kLN) {
        float m = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) m += part[j];
        m /= static_cast<float>(kHidden);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float sq = 0.f;
#pragma unroll
          for (int i = 0; i < 5; ++i) {
            const float d = v[j][i] - m;
            sq = fmaf(d, d, sq);
          }
          part[j] = warp_sum(sq);
        }
        float var = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) var += part[j];
        const float inv = rsqrtf(var / static_cast<float>(kHidden) + p.eps);
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
          for (int i = 0; i < 5; ++i) {
            const int k = 32 * j + lane + 256 * i;
            const half y = __float2half(ln_apply(v[j][i], m, inv, ln_g[k], ln_b[k]));
            yc[k] = y;
            v[j][i] = __half2float(y);
          }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
          for (int i = 0; i < 5; ++i) yc[32 * j + lane + 256 * i] = __float2half(v[j][i]);
      }
      float mx = 0.f, sm = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int i = 0; i < 5; ++i) {
          mx = fmaxf(mx, fabsf(v[j][i]));
          sm += fabsf(v[j][i]);
        }
      mx = warp_max(mx);
      sm = warp_sum(sm);
      const float xinv = mx > 0.f ? kXqMax / mx : 0.f;
      if (lane == 0) {
        xstat[c][0][0] = mx > 0.f ? mx / kXqMax : 0.f;
        xstat[c][1][0] = sm * 1.0001f;  // covers the fp32 rounding of the sum
      }
#pragma unroll
      for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int i = 0; i < 5; ++i) put_xq(c, 32 * j + lane + 256 * i, v[j][i], xinv);
    }
  }
  fence_proxy_async_shared();  // B written by the generic proxy, read by the tensor core
  __syncthreads();
  if constexpr (kClips > 1) {
#pragma unroll
    for (int c = 0; c < kClips; ++c) {
      sx[c] = c < C ? xstat[c][0][0] : 0.f;
      nx1[c] = c < C ? xstat[c][1][0] : 0.f;
    }
  }

  const uint8_t* maskc[kClips];
#pragma unroll
  for (int c = 0; c < kClips; ++c) {
    maskc[c] = msk[0];
    if (kFinalize && c < C && p.first_mask && p.prompt_len > 0 && p.state[2 * c] == p.prompt_len - 1) maskc[c] = msk[1];
  }

  // ---- pass 1: int8 tensor-core GEMV, bounds per row and clip ----
  float lmax[kClips], bmax[kClips];
#pragma unroll
  for (int c = 0; c < kClips; ++c) {
    lmax[c] = -INFINITY;
    bmax[c] = 0.f;
  }
  if (warp == 0) {
    if (lane == 0) {
      const uint64_t policy = policy_evict_first();
      for (int it = S::kStages; it < total; ++it) {
        const int s = it % S::kStages;
        if (!mbar_wait(&empty[s], ((it / S::kStages) & 1) ^ 1)) {
          flag_error(FW_DEVERR_TIMEOUT);
          break;
        }
        issue(it, policy);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_s8(kQTileRows, S::kN);
      const uint32_t xaddr = smem_u32(xb);
      bool ok = true;
      for (int t = 0; t < n_tiles && ok; ++t) {
        const int buf = t & 1;
        if (t >= 2 && !mbar_wait(&acc_empty[buf], ((t >> 1) - 1) & 1)) {
          flag_error(FW_DEVERR_TIMEOUT);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(buf * S::kN);
        for (int c = 0; c < kQChunks; ++c) {
          const int it = t * kQChunks + c, s = it % S::kStages;
          if (!mbar_wait(&full[s], (it / S::kStages) & 1)) {
            flag_error(FW_DEVERR_TIMEOUT);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = sw128_desc(base + s * kQStageBytes);
          const uint64_t bdesc = sw128_desc(xaddr + c * S::kN * kQChunk);
#pragma unroll
          for (int kk = 0; kk < kQChunk / 32; ++kk)
            tc_mma_i8(d, adesc + 2 * kk, bdesc + 2 * kk, idesc, (c | kk) != 0 ? 1u : 0u);
          tc_commit(&empty[s]);
        }
        tc_commit(&acc_full[buf]);
      }
    }
  } else if (warp < 6) {
    const int q = warp & 3;  // TMEM lanes 32q..32q+31 = tile rows 32q..32q+31
    for (int t = 0; t < n_tiles; ++t) {
      const int buf = t & 1;
      if (!mbar_wait_warp(&acc_full[buf], (t >> 1) & 1)) {
        flag_error(FW_DEVERR_TIMEOUT);
        break;
      }
      tc_fence_after();
      uint32_t vv[kClips == 1 ? 2 : 16];
      const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * S::kN);
      if constexpr (kClips == 1) {
        tc_ld2(taddr, vv[0], vv[1]);
      } else {
        tc_ld16(taddr, vv);
      }
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      const int li = t * kQTileRows + q * 32 + lane;
      const bool row_ok = li < nrows;
      const float4 prm = row_ok ? rps[li] : make_float4(0.f, 0.f, 0.f, 0.f);
      bool fetch = false;
#pragma unroll
      for (int c = 0; c < kClips; ++c) {
        if (c >= C) break;
        const int sum = 128 * static_cast<int>(vv[2 * c]) + static_cast<int>(vv[2 * c + 1]);  // exact
        const float approx = prm.x * sx[c] * static_cast<float>(sum);
        const float b = (nx1[c] * prm.y + sx[c] * prm.z + 4e-7f * fabsf(approx)) * 1.00001f + 1e-30f;
        const bool live = row_ok && !maskc[c][li];
        if (row_ok) ub[c * kLmMaxRowsPerCta + li] = live ? approx + b : -INFINITY;
        const float lo = live ? approx - b : -INFINITY;
        if (live) {
          lmax[c] = fmaxf(lmax[c], lo);
          bmax[c] = fmaxf(bmax[c], b);
          if (!isfinite(approx) || !isfinite(b)) bmax[c] = INFINITY;
        }
        // Rows that may survive the selection (against the lower bounds seen so far) have their fp16
        // row fetched into L2 now, so the exact pass reads them from L2. A hint only. With several
        // clips the running maximum is updated once per warp (the lanes' own maximum first) so that
        // 32 lanes do not serialise on the same shared-memory word.
        float run;
        if constexpr (kClips == 1) {
          run = live ? fmaxf(ordered_to_float(atomicMax(&s_lo_max[c], float_to_ordered(lo))), lo) : lo;
        } else {
          // (s_lo_max then ends as this CTA's maximum lower bound of the clip, T; the bound
          // maximum goes to s_b_max the same way, so no reduction is left after the loop)
          const float wlo = warp_max(lo);
          const float wb = warp_max(live ? ((!isfinite(approx) || !isfinite(b)) ? INFINITY : b) : 0.f);
          unsigned prev = 0;
          if (lane == 0) {
            prev = atomicMax(&s_lo_max[c], float_to_ordered(wlo));
            atomicMax(&s_b_max[c], float_to_ordered(wb));
          }
          prev = __shfl_sync(0xffffffffu, prev, 0);
          run = fmaxf(ordered_to_float(prev), wlo);
        }
        if (live && approx + b >= run - (0x1p-9f * (fabsf(run) + 2.f * b) + 0x1p-23f)) fetch = true;
      }
      if (fetch) l2_prefetch(p.w + static_cast<size_t>(r0 + li) * kHidden, kHidden * 2);
    }
  }
  if constexpr (kClips == 1) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      lmax[0] = fmaxf(lmax[0], __shfl_xor_sync(0xffffffffu, lmax[0], o));
      bmax[0] = fmaxf(bmax[0], __shfl_xor_sync(0xffffffffu, bmax[0], o));
    }
    if (lane == 0) {
      warp_l[0][warp] = lmax[0];
      warp_b[0][warp] = bmax[0];
    }
  }
  __syncthreads();

  // ---- row selection per clip: U_r >= T - m (every row when the bound is unusable) ----
  if constexpr (kClips == 1) {
    float t = -INFINITY, bm = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      t = fmaxf(t, warp_l[0][i]);
      bm = fmaxf(bm, warp_b[0][i]);
    }
    const bool all_rows = !(fabsf(t) < 32768.f) || !(bm < 32768.f);
    const float thr = t - (0x1p-9f * (fabsf(t) + 2.f * bm) + 0x1p-23f);
    // compacted with a ballot: one shared atomic per warp and 32 rows (the rescoring order does not
    // matter, the packed keys are max-reduced)
    for (int i0 = warp * 32; i0 < nrows; i0 += 256) {
      const int i = i0 + lane;
      const bool take = i < nrows && !maskc[0][i] && (all_rows || ub[i] >= thr);
      const unsigned bal = __ballot_sync(0xffffffffu, take);
      int base = 0;
      if (lane == 0 && bal) base = atomicAdd(&ncand[0], __popc(bal));
      base = __shfl_sync(0xffffffffu, base, 0);
      if (take) cand[base + __popc(bal & ((1u << lane) - 1u))] = static_cast<unsigned short>(i);
    }
  } else if (warp < C) {  // warp w selects clip w's rows, compacted with a ballot (no atomics)
    const int c = warp;
    const float t = ordered_to_float(s_lo_max[c]), bm = ordered_to_float(s_b_max[c]);
    const bool all_rows = !(fabsf(t) < 32768.f) || !(bm < 32768.f);
    const float thr = t - (0x1p-9f * (fabsf(t) + 2.f * bm) + 0x1p-23f);
    const uint8_t* mk = (kFinalize && p.first_mask && p.prompt_len > 0 && p.state[2 * c] == p.prompt_len - 1)
                            ? msk[1] : msk[0];
    int n = 0;
    for (int i0 = 0; i0 < nrows; i0 += 32) {
      const int i = i0 + lane;
      const bool take = i < nrows && !mk[i] && (all_rows || ub[c * kLmMaxRowsPerCta + i] >= thr);
      const unsigned bal = __ballot_sync(0xffffffffu, take);
      if (take) cand[c * kLmMaxRowsPerCta + n + __popc(bal & ((1u << lane) - 1u))] = static_cast<unsigned short>(i);
      n += __popc(bal);
    }
    if (lane == 0) ncand[c] = n;
  }
  __syncthreads();

  // ---- pass 2: exact fp16 logits of the surviving rows, four rows per warp at a time; with several
  // clips, warp w rescores clip w's survivors (the 8 warps work on the 8 clips in parallel) ----
  static_assert(kClips == 1 || kClips == 8, "pass 2 maps warp w to clip w");
  if (kClips > 1 && lane == 0) {
#pragma unroll
    for (int c = 0; c < kClips; ++c) warp_best[c][warp] = 0ull;  // this warp's entry of every clip
  }
  if (kClips == 1 || warp < C) {
    const int c = kClips == 1 ? 0 : warp;
    float xf[40];
    load_x40(ys + c * kHidden, xf);
    const int nc = ncand[c];
    const unsigned short* cl = cand + c * kLmMaxRowsPerCta;
    unsigned long long mine = 0;
    const int j0 = kClips == 1 ? 4 * warp : 0, jstep = kClips == 1 ? 32 : 4;
    for (int j = j0; j < nc; j += jstep) {
      int rr[4];
      const half* rows[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        rr[q] = r0 + cl[min(j + q, nc - 1)];  // a repeated row repeats its key
        rows[q] = p.w + static_cast<size_t>(rr[q]) * kHidden;
      }
      float acc[4];
      dot1280_ptrs<4>(rows, xf, acc);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const unsigned long long k = pack_score(round_half(acc[q]), rr[q]);
        mine = k > mine ? k : mine;
      }
    }
    if (lane == 0) warp_best[c][warp] = mine;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, S::kTmemCols);
  }
  if (threadIdx.x == 0) {
    for (int c = 0; c < C; ++c) {
      unsigned long long m = 0;
      for (int i = 0; i < 8; ++i) m = warp_best[c][i] > m ? warp_best[c][i] : m;
      if (m) atomicMax(p.best + c, m);
    }
    if (kFinalize) {  // the acq_rel arrival releases this CTA's maxima and, in the last CTA, acquires all
      if (atomic_add_acq_rel(p.counter, 1u) == gridDim.x - 1) {
        for (int c = 0; c < C; ++c) {
          const unsigned long long b = atomicExch(p.best + c, 0ull);
          finalize_token(b, p.tokens + c * p.tokens_stride, p.n_tokens, p.state + 2 * c, p.cur + c, p.max_pos,
                         p.prompt_len);
        }
        *p.counter = 0u;
      }
    }
  }
}

// One warp per vocab row: int8 row, scale and the two error terms of lm_head_q_kernel.
__global__ void __launch_bounds__(256) lm_quantize_kernel(const half* __restrict__ w, int vocab,
                                                          int8_t* __restrict__ wq, float4* __restrict__ rp) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= vocab) return;
  const half* wr = w + static_cast<size_t>(row) * kHidden;
  float v[40];
#pragma unroll
  for (int c = 0; c < 5; ++c) {
    const uint4 u = reinterpret_cast<const uint4*>(wr)[lane + 32 * c];
    const half2* h2 = reinterpret_cast<const half2*>(&u);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __half22float2(h2[k]);
      v[8 * c + 2 * k] = f.x;
      v[8 * c + 2 * k + 1] = f.y;
    }
  }
  float wmax = 0.f;
#pragma unroll
  for (int i = 0; i < 40; ++i) wmax = fmaxf(wmax, fabsf(v[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) wmax = fmaxf(wmax, __shfl_xor_sync(0xffffffffu, wmax, o));
  const float s = wmax > 0.f ? wmax / 127.f : 1.f;
  double err = 0.0;
  int q1 = 0;
  int8_t q[40];
#pragma unroll
  for (int i = 0; i < 40; ++i) {
    const int qi = max(-127, min(127, __float2int_rn(v[i] / s)));
    q[i] = static_cast<int8_t>(qi);
    q1 += abs(qi);
    err = fmax(err, fabs(static_cast<double>(v[i]) - static_cast<double>(qi) * static_cast<double>(s)));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    err = fmax(err, __shfl_xor_sync(0xffffffffu, err, o));
    q1 += __shfl_xor_sync(0xffffffffu, q1, o);
  }
#pragma unroll
  for (int c = 0; c < 5; ++c) {
    uint2 packed;
    packed.x = (static_cast<uint32_t>(static_cast<uint8_t>(q[8 * c + 0]))) |
               (static_cast<uint32_t>(static_cast<uint8_t>(q[8 * c + 1])) << 8) |
               (static_cast<uint32_t>(static_cast<uint8_t>(q[8 * c + 2])) << 16) |
               (static_cast<uint32_t>(static_cast<uint8_t>(q[8 * c + 3])) << 24);
    packed.y = (static_cast<uint32_t>(static_cast<uint8_t>(q[8 * c + 4]))) |
               (static_cast<uint32_t>(static_cast<uint8_t>(q[8 * c + 5])) << 8) |
               (static_cast<uint32_t>(static_cast<uint8_t>(q[8 * c + 6])) << 16) |
               (static_cast<uint32_t>(static_cast<uint8_t>(q[8 * c + 7])) << 24);
    reinterpret_cast<uint2*>(wq + static_cast<size_t>(row) * kHidden)[lane + 32 * c] = packed;
  }
  if (lane == 0) {
    const double a = err + 1e-5 * static_cast<double>(wmax);
    const double c2 = 0.51 * static_cast<double>(s) * static_cast<double>(q1);
    rp[row] = make_float4(s, __double2float_ru(a), __double2float_ru(c2), 0.f);
  }
}

__global__ void argmax_finalize_kernel(unsigned long long* best, int64_t* tokens, int64_t n_tokens, int64_t* state,
                                       int64_t* cur, int max_pos) {
  pdl_wait();
  pdl_trigger();
  const unsigned long long b = *best;
  *best = 0;
  finalize_token(b, tokens, n_tokens, state, cur, max_pos, 0);
}

// ---------------------------------------------------------------------------------------------
// LayerNorm-prologue GEMV: out[r] = act(W[r] . LN(h) + b[r]) for this CTA's rows. Everything the
// kernel reads that no in-flight launch writes is fetched before the PDL wait: the CTA's weight
// rows (rows_per_cta x 1280 fp16) by bulk copy into shared memory, the LayerNorm gamma/beta and the
// bias entries into registers. After the wait the only global round trip is the read of h.
struct GemvParams {
  const half* w;
  const half* b;
  half* out;
  int n_out;
  int k;
  int rows_per_cta;
  // LayerNorm prologue
  const half* h;
  const half* gamma;
  const half* beta;
  float eps;
  // residual GEMV
  const half* x;
  half* h_res;
  // deferred residual (ln_gemv_kernel<.., .., true>, a launch in clusters of kHeadCtas): the LayerNorm
  // input is h + fp16(sum over heads of res_part + res_bias), formed as head_block_kernel does, and
  // written to h_out by the first cluster
  const float* res_part;
  const half* res_bias;
  half* h_out;
};

// kRowsPerWarp = rows_per_cta / 8 (1, 3 or 4): warp w owns rows w, w + 8, ...
template <int kAct, int kRowsPerWarp, bool kRes = false>
__global__ void __launch_bounds__(256) ln_gemv_kernel(GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bar, bar_h;
  __shared__ float red[16];
  __shared__ __align__(16) half ys[kHidden];
  __shared__ __align__(16) half hres[kRes ? kHidden : 8];  // the formed LayerNorm input (kRes)
  const int crank = kRes ? static_cast<int>(blockIdx.x % kHeadCtas) : 0;  // rank in the cluster
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r0 = blockIdx.x * p.rows_per_cta;
  const int nr = min(p.rows_per_cta, p.n_out - r0);
  half* ws = reinterpret_cast<half*>(smem);

  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    if (kRes) mbar_init(&bar_h, 1);
    mbar_fence_init();
    if (kRes) mbar_arrive_expect_tx(&bar_h, (kHeadCtas - 1) * kOutRows * 2);  // the other CTAs' rows
    if (nr > 0) {
      mbar_arrive_expect_tx(&bar, static_cast<unsigned>(nr) * kHidden * 2);
      for (int r = 0; r < nr; ++r)
        bulk_g2s_stream(ws + r * kHidden, p.w + static_cast<size_t>(r0 + r) * kHidden, kHidden * 2, &bar,
                        policy_evict_first());
    }
  }
  float g[5], be[5], bias[kRowsPerWarp];
#pragma unroll
  for (int i = 0; i < 5; ++i) {
    g[i] = __half2float(p.gamma[threadIdx.x + i * 256]);
    be[i] = __half2float(p.beta[threadIdx.x + i * 256]);
  }
#pragma unroll
  for (int i = 0; i < kRowsPerWarp; ++i) {
    const int r = warp + 8 * i;
    bias[i] = (p.b && r < nr) ? __half2float(p.b[r0 + r]) : 0.f;
  }
  __syncthreads();
  if (kRes) cluster_arrive_relaxed();  // completed before the first DSMEM store
  // Released before the wait: the next launch (fc2 in the decode step) reads only weights before its
  // own wait, so it may start its weight copies while the launch before this one still runs.
  pdl_trigger();
  pdl_wait();

  float v[5];
  if constexpr (kRes) {
    // rows crank*160 .. +159 of h + fp16(sum over heads, in order, of res_part + res_bias), then those
    // rows to the cluster's other CTAs (head_block_kernel's residual exchange)
    const int tid = threadIdx.x;
    cluster_wait();
    if (tid < kOutRows) {
      const int e = crank * kOutRows + tid;
      float pv[kHeads];
#pragma unroll
      for (int hh = 0; hh < kHeads; ++hh) pv[hh] = __ldcg(p.res_part + static_cast<size_t>(hh) * kHidden + e);
      const float h0 = __half2float(p.h[e]), rb = __half2float(p.res_bias[e]);
      float acc = 0.f;
#pragma unroll
      for (int hh = 0; hh < kHeads; ++hh) acc += pv[hh];
      const half hv = __float2half(h0 + round_half(acc + rb));
      hres[e] = hv;
      if (blockIdx.x < kHeadCtas) p.h_out[e] = hv;  // the first cluster materialises it (fc2's residual)
    }
    __syncthreads();
    constexpr int kChunks = kOutRows * 2 / 16;
    if (tid < (kHeadCtas - 1) * kChunks) {
      const int dst = tid / kChunks + (tid / kChunks >= crank ? 1 : 0), c = tid % kChunks;
      const uint4 val = reinterpret_cast<const uint4*>(hres + crank * kOutRows)[c];
      st_async_v4(cluster_map(hres + crank * kOutRows, dst) + 16 * c, val, cluster_map(&bar_h, dst));
    }
    if (!mbar_wait_cluster(&bar_h, 0)) flag_error(FW_DEVERR_TIMEOUT);
    cluster_arrive_relaxed();  // every CTA has received its rows once all have arrived (the wait at exit)
#pragma unroll
    for (int i = 0; i < 5; ++i) v[i] = __half2float(hres[tid + i * 256]);
  } else {
#pragma unroll
    for (int i = 0; i < 5; ++i) v[i] = __half2float(p.h[threadIdx.x + i * 256]);
  }
  float mean, inv;
  ln1280_stats(v, red, p.eps, mean, inv);
#pragma unroll
  for (int i = 0; i < 5; ++i) ys[threadIdx.x + i * 256] = __float2half(ln_apply(v[i], mean, inv, g[i], be[i]));
  __syncthreads();
  float xf[40];
  load_x40(ys, xf);
  if (nr > 0 && !mbar_wait(&bar, 0)) flag_error(FW_DEVERR_TIMEOUT);
  if (nr == 8 * kRowsPerWarp) {  // full CTA: all rows interleaved
    float acc[kRowsPerWarp];
    dot1280_rows<kRowsPerWarp>(ws + warp * kHidden, 8 * kHidden, xf, acc);
    if (lane < kRowsPerWarp) {  // lane i finishes row warp + 8 i
      float a = acc[0], bi = bias[0];
#pragma unroll
      for (int i = 1; i < kRowsPerWarp; ++i)
        if (lane == i) {
          a = acc[i];
          bi = bias[i];
        }
      float o = round_half(a + bi);
      if (kAct == 1) o = gelu_erf(o);
      p.out[r0 + warp + 8 * lane] = __float2half(o);
    }
  } else {  // ragged last CTA
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
      const int r = warp + 8 * i;
      if (r < nr) {
        const float acc = warp_sum(dot1280_lane(reinterpret_cast<const uint4*>(ws + r * kHidden), xf));
        if (lane == 0) {
          float o = round_half(acc + bias[i]);
          if (kAct == 1) o = gelu_erf(o);
          p.out[r0 + r] = __float2half(o);
        }
      }
    }
  }
  if (kRes) cluster_wait();
}

// Residual GEMV: h[r] = fp16(h[r] + fp16(W[r] . x + b[r])) for this CTA's kResidRows rows, x of
// length k = 256 * kChunks. The CTA splits k, not rows: thread t owns 16-byte chunks t, t + 320, ...
// of x (in registers) and of every row, accumulates one partial per row, and the partials are summed
// over each warp (xor tree) and then over the warps in order, so each weight and x byte is read
// from shared memory once. The weight rows are bulk-copied and the bias loaded before the PDL wait,
// the residual entries after it.
constexpr int kResidRows = 10;  // 1280 / 10 = 128 CTAs: no SM holds two, leaving room for the next launch
constexpr int kResidThreads = 320;

template <int kChunks>
__global__ void __launch_bounds__(kResidThreads) gemv_residual_kernel(GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bar;
  __shared__ float red[kResidThreads / 32][kResidRows];
  constexpr int k = 256 * kChunks;
  constexpr int kc = k / 8;                                            // 16-byte chunks per row
  constexpr int kPer = (kc + kResidThreads - 1) / kResidThreads;       // chunks per thread
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r0 = blockIdx.x * kResidRows;
  const int nr = min(kResidRows, p.n_out - r0);
  const uint4* ws = reinterpret_cast<const uint4*>(smem);

  if (tid == 0) {
    mbar_init(&bar, 1);
    mbar_fence_init();
    if (nr > 0) {
      mbar_arrive_expect_tx(&bar, static_cast<unsigned>(nr) * k * 2);
      for (int r = 0; r < nr; ++r)
        bulk_g2s_stream(smem + static_cast<size_t>(r) * k * 2, p.w + static_cast<size_t>(r0 + r) * k, k * 2, &bar,
                        policy_evict_first());
    }
  }
  const bool owner = tid < nr;  // thread r finishes row r
  const float bias = (p.b && owner) ? __half2float(p.b[r0 + tid]) : 0.f;
  __syncthreads();
  // Released before the wait (the next decode launch reads only weights, and cache rows of earlier
  // steps, before its own wait); the residual is read after it.
  pdl_trigger();
  pdl_wait();
  const float hres = owner ? __half2float(p.h_res[r0 + tid]) : 0.f;
  uint4 xv[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int c = tid + kResidThreads * j;
    xv[j] = c < kc ? reinterpret_cast<const uint4*>(p.x)[c] : make_uint4(0, 0, 0, 0);
  }
  if (nr > 0 && !mbar_wait(&bar, 0)) flag_error(FW_DEVERR_TIMEOUT);
  float acc[kResidRows];
#pragma unroll
  for (int r = 0; r < kResidRows; ++r) acc[r] = 0.f;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int c = tid + kResidThreads * j;
    if (c < kc) {
      const half2* px = reinterpret_cast<const half2*>(&xv[j]);
#pragma unroll
      for (int r = 0; r < kResidRows; ++r) {
        if (r < nr) {
          const uint4 wv = ws[r * kc + c];
          const half2* pw = reinterpret_cast<const half2*>(&wv);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 fw = __half22float2(pw[e]), fx = __half22float2(px[e]);
            acc[r] = fmaf(fw.x, fx.x, acc[r]);
            acc[r] = fmaf(fw.y, fx.y, acc[r]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int r = 0; r < kResidRows; ++r) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < kResidRows; ++r) red[warp][r] = acc[r];
  }
  __syncthreads();
  if (owner) {
    float sum = 0.f;
#pragma unroll
    for (int w = 0; w < kResidThreads / 32; ++w) sum += red[w][tid];
    p.h_res[r0 + tid] = __float2half(hres + round_half(sum + bias));
  }
}

// ---------------------------------------------------------------------------------------------
// Stand-alone ops.
__global__ void embed_pos_kernel(const half* __restrict__ embed, const half* __restrict__ pos_embed,
                                 const int64_t* __restrict__ ids, const int64_t* __restrict__ positions,
                                 half* __restrict__ out, int n, int vocab, int max_pos, int hidden) {
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x;
  if (row >= n) return;
  int64_t id = ids[row], pos = positions[row];
  if (id < 0 || id >= vocab || pos < 0 || pos >= max_pos) {
    if (threadIdx.x == 0) flag_error(FW_DEVERR_BAD_INDEX);
    id = id < 0 ? 0 : (id >= vocab ? vocab - 1 : id);
    pos = pos < 0 ? 0 : (pos >= max_pos ? max_pos - 1 : pos);
  }
  const half2* e = reinterpret_cast<const half2*>(embed + static_cast<size_t>(id) * hidden);
  const half2* q = reinterpret_cast<const half2*>(pos_embed + static_cast<size_t>(pos) * hidden);
  half2* o = reinterpret_cast<half2*>(out + static_cast<size_t>(row) * hidden);
  for (int i = threadIdx.x; i < hidden / 2; i += blockDim.x) {
    const float2 a = __half22float2(e[i]), b = __half22float2(q[i]);
    o[i] = __floats2half2_rn(a.x + b.x, a.y + b.y);
  }
}

__global__ void gelu_kernel(const half* __restrict__ x, half* __restrict__ y, int64_t n) {
  pdl_wait();
  pdl_trigger();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += stride)
    y[i] = __float2half(gelu_erf(__half2float(x[i])));
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, v, o);
    v = other > v ? other : v;
  }
  return v;
}

__global__ void __launch_bounds__(256) argmax_f16_kernel(const half* __restrict__ logits, int64_t n,
                                                         const bool* __restrict__ suppress,
                                                         unsigned long long* __restrict__ key) {
  __shared__ unsigned long long wb[8];
  pdl_wait();
  pdl_trigger();
  unsigned long long mine = 0;
  const int64_t n8 = n / 8;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t c = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; c < n8; c += stride) {
    const uint4 v = reinterpret_cast<const uint4*>(logits)[c];
    const half* hv = reinterpret_cast<const half*>(&v);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t i = c * 8 + j;
      if (suppress && suppress[i]) continue;
      const unsigned long long k = pack_score(__half2float(hv[j]), static_cast<int>(i));
      mine = k > mine ? k : mine;
    }
  }
  for (int64_t i = n8 * 8 + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += stride) {
    if (suppress && suppress[i]) continue;
    const unsigned long long k = pack_score(__half2float(logits[i]), static_cast<int>(i));
    mine = k > mine ? k : mine;
  }
  mine = warp_max_u64(mine);
  if ((threadIdx.x & 31) == 0) wb[threadIdx.x >> 5] = mine;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long m = 0;
    for (int i = 0; i < 8; ++i) m = wb[i] > m ? wb[i] : m;
    if (m) atomicMax(key, m);
  }
}

__global__ void argmax_index_kernel(unsigned long long* key, int64_t* out_index) {
  pdl_wait();
  pdl_trigger();
  const unsigned long long k = *key;
  *key = 0ull;
  *out_index = k ? static_cast<int64_t>(unpack_index(k)) : -1;
}

// ---------------------------------------------------------------------------------------------
// Batched decode: one decode step for `clips` independent clips (at most kMaxClips) per weight read.
// Each clip has its own residual stream, caches, position and tokens; the weights are streamed once
// per step for all of them. Every per-clip value is computed with exactly the arithmetic of the
// batch-1 step above (the same LayerNorm summation order, the same per-lane dot-product chains and
// warp xor-trees, the same split attention and combine, the same head-ordered output-projection
// sum, the same LM-head key), so each clip's tokens are bit-identical to decoding it alone.
constexpr int kMaxClips = 8;

struct BatchGemvParams {
  const half* w;  // [n_out, 1280]
  const half* b;  // [n_out] or null
  half* out;      // clip c's outputs at out + c * out_stride
  int n_out, out_stride, clips;
  const half* h;  // [clips, 1280] LayerNorm input
  const half* gamma;
  const half* beta;
  float eps;
  // layer 0: h_c = fp16(embed[token_c] + pos_embed[position_c]), written to h_out by CTA 0
  const half* embed;
  const half* pos_embed;
  const int64_t* cur;    // [clips]
  const int64_t* state;  // [clips, 2]
  const int64_t* prompt;
  int prompt_len, vocab, max_pos;
  half* h_out;
};

// LayerNorm (+ optional GELU epilogue) GEMV for every clip: out_c[r] = act(W[r] . LN(h_c) + b[r]).
// 512 threads: the two halves of the CTA handle clips 0-3 and 4-7. Each half computes its clips'
// LayerNorm exactly as a 256-thread add_layernorm_kernel does (ln1280_stats order) and stores the
// normalised rows as fp32 (exact fp16 values) in two planes per clip, elements 0-3 and 4-7 of every
// 8-element chunk, so a lane's float4 reads of its chunk are consecutive across the warp. The CTA's
// 8 * kRowsPerWarp weight rows are bulk-copied into shared memory before the PDL wait. Warp w of a
// half owns rows w, w + 8, ...: per 16-byte chunk it converts each of its rows' chunk to fp32 once and
// runs the fma chains of its four clips (the lane order of dot1280_lane), then the warp xor-tree.
constexpr int kBlnThreads = 512;

template <int kRowsPerWarp>
struct BlnShape {
  static constexpr int kRows = 8 * kRowsPerWarp;
  static constexpr int kWBytes = kRows * kHidden * 2;
  static constexpr int kSmem = kWBytes + kMaxClips * kHidden * 4;
};

template <int kAct, int kRowsPerWarp, bool kEmbed>
__global__ void __launch_bounds__(kBlnThreads, 1) bln_gemv_kernel(BatchGemvParams p) {
  using S = BlnShape<kRowsPerWarp>;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bar;
  __shared__ float red[kMaxClips][16];
  half* ws = reinterpret_cast<half*>(smem);
  float4* xs = reinterpret_cast<float4*>(smem + S::kWBytes);  // clip c: plane A [160], plane B [160]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int half_id = warp >> 3, wr = warp & 7, t256 = tid & 255;
  const int r0 = blockIdx.x * S::kRows;
  const int nr = min(S::kRows, p.n_out - r0);
  const int C = p.clips;
  const int c0 = 4 * half_id;  // this half's clips c0 .. c0 + 3
  if (tid == 0) {
    mbar_init(&bar, 1);
    mbar_fence_init();
    if (nr > 0) {
      mbar_arrive_expect_tx(&bar, static_cast<unsigned>(nr) * kHidden * 2);
      const uint64_t pol = policy_evict_first();
      for (int r = 0; r < nr; ++r)
        bulk_g2s_stream(ws + r * kHidden, p.w + static_cast<size_t>(r0 + r) * kHidden, kHidden * 2, &bar, pol);
    }
  }
  float g[5], be[5], bias[kRowsPerWarp];
#pragma unroll
  for (int i = 0; i < 5; ++i) {
    g[i] = __half2float(p.gamma[t256 + i * 256]);
    be[i] = __half2float(p.beta[t256 + i * 256]);
  }
#pragma unroll
  for (int i = 0; i < kRowsPerWarp; ++i) {
    const int r = wr + 8 * i;
    bias[i] = (p.b && r < nr) ? __half2float(p.b[r0 + r]) : 0.f;
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();

  // LayerNorm of this half's clips, thread t256 holding elements t256 + 256 i as in ln1280_stats
  float v[4][5];
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    const int c = c0 + cc;
    if (c >= C) break;
    if (kEmbed) {
      const int64_t raw = p.state[2 * c];
      const int pos = static_cast<int>(min(max(raw, int64_t(0)), int64_t(p.max_pos - 1)));
      int64_t tok = pos < p.prompt_len ? p.prompt[pos] : p.cur[c];
      if (raw < 0 || raw >= p.max_pos || tok < 0 || tok >= p.vocab) {
        if (t256 == 0 && blockIdx.x == 0) flag_error(FW_DEVERR_BAD_INDEX);
        tok = tok < 0 ? 0 : (tok >= p.vocab ? p.vocab - 1 : tok);
      }
      const half* er = p.embed + static_cast<size_t>(tok) * kHidden;
      const half* pr = p.pos_embed + static_cast<size_t>(pos) * kHidden;
#pragma unroll
      for (int i = 0; i < 5; ++i) {
        v[cc][i] = round_half(__half2float(er[t256 + i * 256]) + __half2float(pr[t256 + i * 256]));
        if (blockIdx.x == 0) p.h_out[c * kHidden + t256 + i * 256] = __float2half(v[cc][i]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 5; ++i) v[cc][i] = __half2float(p.h[c * kHidden + t256 + i * 256]);
    }
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < 5; ++i) sum += v[cc][i];
    sum = warp_sum(sum);
    if (lane == 0) red[c][wr] = sum;
  }
  __syncthreads();
  float mean[4];
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    const int c = c0 + cc;
    if (c >= C) break;
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) m += red[c][i];
    m /= static_cast<float>(kHidden);
    mean[cc] = m;
    float sq = 0.f;
#pragma unroll
    for (int i = 0; i < 5; ++i) {
      const float d = v[cc][i] - m;
      sq = fmaf(d, d, sq);
    }
    sq = warp_sum(sq);
    if (lane == 0) red[c][8 + wr] = sq;
  }
  __syncthreads();
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    const int c = c0 + cc;
    if (c >= C) break;
    float var = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) var += red[c][8 + i];
    const float inv = rsqrtf(var / static_cast<float>(kHidden) + p.eps);
    float* plane = reinterpret_cast<float*>(xs + c * 2 * (kHidden / 8));
#pragma unroll
    for (int i = 0; i < 5; ++i) {
      const int k = t256 + i * 256, q = k >> 3, e = k & 7;
      const float y = __half2float(__float2half(ln_apply(v[cc][i], mean[cc], inv, g[i], be[i])));
      plane[(e < 4 ? q : (kHidden / 8) + q) * 4 + (e & 3)] = y;
    }
  }
  __syncthreads();
  if (nr > 0 && !mbar_wait(&bar, 0)) flag_error(FW_DEVERR_TIMEOUT);

  float acc[kRowsPerWarp][4];
#pragma unroll
  for (int i = 0; i < kRowsPerWarp; ++i)
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) acc[i][cc] = 0.f;
#pragma unroll
  for (int ch = 0; ch < 5; ++ch) {
    float wf[kRowsPerWarp][8];
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
      const uint4 wv = reinterpret_cast<const uint4*>(ws + (wr + 8 * i) * kHidden)[lane + 32 * ch];
      const half2* h2 = reinterpret_cast<const half2*>(&wv);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(h2[k]);
        wf[i][2 * k] = f.x;
        wf[i][2 * k + 1] = f.y;
      }
    }
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      const int c = c0 + cc;
      if (c >= C) break;
      const float4 xa = xs[c * 2 * (kHidden / 8) + lane + 32 * ch];
      const float4 xb = xs[c * 2 * (kHidden / 8) + (kHidden / 8) + lane + 32 * ch];
      const float x8[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
      for (int i = 0; i < kRowsPerWarp; ++i)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[i][cc] = fmaf(wf[i][e], x8[e], acc[i][cc]);
    }
  }
#pragma unroll
  for (int i = 0; i < kRowsPerWarp; ++i) {
    const int r = wr + 8 * i;
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      const int c = c0 + cc;
      if (c >= C) break;
      const float a = warp_sum(acc[i][cc]);
      if (lane == cc && r < nr) {
        float o = round_half(a + bias[i]);
        if (kAct == 1) o = gelu_erf(o);
        p.out[static_cast<size_t>(c) * p.out_stride + r0 + r] = __float2half(o);
      }
    }
  }
}

// Output projection of the attention heads + bias + residual for every clip:
// h_c[r] = fp16(h_c[r] + fp16(sum_head (W_o[head][r] . o_c[head]) + b[r])) with W_o head-major
// [heads, 1280, 64]. Per (row, head) the dot is the two-chain rotated-chunk order of
// head_block_kernel's output-projection partial (chunk (j + r) mod 8 at step j, even and odd steps in
// separate chains), and the head sum runs in head order, so the result equals head_block_kernel's.
// A CTA owns kOutRowsB = 16 rows; its slice of every head (16 x 64 fp16) is bulk-copied into shared
// memory before the PDL wait. Thread (k, clip pair, head pair) computes rows r0 + k and r0 + k + 8 (the
// same rotation, so each o chunk read serves both rows) for two clips and two heads; the attention
// outputs are staged as fp32 in two planes (elements 0-3 and 4-7 of every chunk) so a warp's float4
// reads are conflict-free. The per-head partials meet in shared memory and are summed in head order.
constexpr int kOutRowsB = 16;                                   // 1280 / 16 = 80 CTAs
constexpr int kOutThreadsB = 320;                               // 8 row pairs x 4 clip pairs x 10 head pairs
constexpr int kBoutWBytes = kHeads * kOutRowsB * kHeadDim * 2;  // 40 KB
constexpr int kBoutSmem = kBoutWBytes + kMaxClips * kHidden * 4 + kOutRowsB * kMaxClips * kHeads * 4;

struct BatchOutParams {
  const half* wo;    // head-major [heads, 1280, 64]
  const half* bo;    // [1280]
  const half* attn;  // [clips, 1280] attention outputs (head-major within a clip)
  half* h;           // [clips, 1280] residual stream, updated in place
  int clips;
};

__global__ void __launch_bounds__(kOutThreadsB, 1) bout_residual_kernel(BatchOutParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const half* ws = reinterpret_cast<const half*>(smem);                    // [heads][16 rows][64]
  float4* os = reinterpret_cast<float4*>(smem + kBoutWBytes);             // clip c: A [160], B [160]
  float* part = reinterpret_cast<float*>(smem + kBoutWBytes + kMaxClips * kHidden * 4);  // [16][8][20]
  __shared__ __align__(8) uint64_t bar;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r0 = blockIdx.x * kOutRowsB;
  const int C = p.clips;
  if (tid == 0) {
    mbar_init(&bar, 1);
    mbar_fence_init();
    mbar_arrive_expect_tx(&bar, kBoutWBytes);
    const uint64_t pol = policy_evict_first();
    for (int hh = 0; hh < kHeads; ++hh)
      bulk_g2s_stream(smem + hh * kOutRowsB * kHeadDim * 2, p.wo + (static_cast<size_t>(hh) * kHidden + r0) * kHeadDim,
                      kOutRowsB * kHeadDim * 2, &bar, pol);
  }
  // epilogue owner: (row, clip) = (tid % 16, tid / 16) for tid < 128
  const bool owner = tid < kOutRowsB * kMaxClips && tid / kOutRowsB < C;
  const float obias = (p.bo && owner) ? __half2float(p.bo[r0 + tid % kOutRowsB]) : 0.f;
  __syncthreads();
  pdl_wait();
  pdl_trigger();
  for (int i = tid; i < C * kHidden; i += kOutThreadsB) {
    const int c = i / kHidden, k = i % kHidden, q = k >> 3, e = k & 7;
    reinterpret_cast<float*>(os + c * 2 * (kHidden / 8))[(e < 4 ? q : (kHidden / 8) + q) * 4 + (e & 3)] =
        __half2float(p.attn[i]);
  }
  __syncthreads();
  if (!mbar_wait(&bar, 0)) flag_error(FW_DEVERR_TIMEOUT);
  const int k = lane & 7, cp = lane >> 3, hp = warp;  // rows r0+k, r0+k+8; clips 2cp, 2cp+1; heads 2hp, 2hp+1
  const int c0 = 2 * cp;
  if (c0 < C) {
    const bool two = c0 + 1 < C;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int hh = 2 * hp + q;
      const uint4* wa = reinterpret_cast<const uint4*>(ws + (hh * kOutRowsB + k) * kHeadDim);
      const uint4* wb = reinterpret_cast<const uint4*>(ws + (hh * kOutRowsB + k + 8) * kHeadDim);
      float acc[2][2][2] = {};  // [row][clip][chain]
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int ch = (j + r0 + k) & 7;  // head_block_kernel's rotation (its row index mod 8 equals r's)
        float w8[2][8];
        const uint4 wva = wa[ch], wvb = wb[ch];
        const half2* a2 = reinterpret_cast<const half2*>(&wva);
        const half2* b2 = reinterpret_cast<const half2*>(&wvb);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 fa = __half22float2(a2[e]), fb = __half22float2(b2[e]);
          w8[0][2 * e] = fa.x;
          w8[0][2 * e + 1] = fa.y;
          w8[1][2 * e] = fb.x;
          w8[1][2 * e + 1] = fb.y;
        }
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          if (cc == 1 && !two) break;
          const int c = c0 + cc;
          const float4 oa = os[c * 2 * (kHidden / 8) + hh * 8 + ch];
          const float4 ob = os[c * 2 * (kHidden / 8) + (kHidden / 8) + hh * 8 + ch];
          const float o8[8] = {oa.x, oa.y, oa.z, oa.w, ob.x, ob.y, ob.z, ob.w};
#pragma unroll
          for (int rr = 0; rr < 2; ++rr) {
            float& a = acc[rr][cc][j & 1];
#pragma unroll
            for (int e = 0; e < 8; ++e) a = fmaf(w8[rr][e], o8[e], a);
          }
        }
      }
#pragma unroll
      for (int rr = 0; rr < 2; ++rr)
#pragma unroll
        for (int cc = 0; cc < 2; ++cc)
          if (cc == 0 || two) part[((k + 8 * rr) * kMaxClips + c0 + cc) * kHeads + hh] = acc[rr][cc][0] + acc[rr][cc][1];
    }
  }
  __syncthreads();
  if (owner) {
    const int rl = tid % kOutRowsB, c = tid / kOutRowsB;
    float acc = 0.f;
#pragma unroll
    for (int hh = 0; hh < kHeads; ++hh) acc += part[(rl * kMaxClips + c) * kHeads + hh];
    half* hr = p.h + static_cast<size_t>(c) * kHidden + r0 + rl;
    *hr = __float2half(__half2float(*hr) + round_half(acc + obias));
  }
}

// Sum of 32 per-lane values v[0..31] over the 32 lanes of a warp, returning in lane l the sum of
// index l: the xor butterfly of warp_sum (distances 16, 8, 4, 2, 1) applied to all 32 values at once,
// each level halving the values a lane keeps (it adds the partner's copy of the half it keeps and
// hands over the other half). Every sum is formed from the same operands in the same tree as
// warp_sum(v[l]), so the result is bit-identical to it; 31 shuffles instead of 160.
__device__ __forceinline__ float warp_sum32_transpose(float (&v)[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int d = 16, n = 16; d > 0; d >>= 1, n >>= 1) {
    const bool up = (lane & d) != 0;
#pragma unroll
    for (int i = 0; i < n; ++i) {
      const float send = up ? v[i] : v[n + i];
      const float keep = up ? v[n + i] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, d);
    }
  }
  return v[0];
}

// fc2 + residual for every clip: h_c[r] = fp16(h_c[r] + fp16(W[r] . x_c + b[r])), x_c = the fc1 output
// [5120] of clip c. Same K split and reduction order as gemv_residual_kernel<20> (thread t owns
// 16-byte chunks t and t + 320 of every row, warp xor-tree, warps summed in order). A CTA owns
// kResidRows rows, bulk-copied into shared memory before the PDL wait; the clips are taken four at a
// time with their x chunks converted to fp32 in registers once, each weight chunk converted once per
// group and used for all four clips. Rows 0-7 of a group are reduced with warp_sum32_transpose.
constexpr int kBfc2Threads = kResidThreads;  // 320

struct BatchFc2Params {
  const half* w;   // [1280, 5120]
  const half* b;   // [1280]
  const half* x;   // [clips, 5120]
  half* h;         // [clips, 1280]
  int clips;
};

__global__ void __launch_bounds__(kBfc2Threads, 1) bfc2_residual_kernel(BatchFc2Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bar;
  __shared__ float red[kBfc2Threads / 32][kResidRows][kMaxClips];
  static_assert(kResidRows == 10, "the transposed reduction covers rows 0-7, rows 8-9 use warp_sum");
  constexpr int kc = kFfn / 8;  // 640 chunks per row; thread t owns chunks t and t + 320
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r0 = blockIdx.x * kResidRows;
  const int C = p.clips;
  const uint4* ws = reinterpret_cast<const uint4*>(smem);
  if (tid == 0) {
    mbar_init(&bar, 1);
    mbar_fence_init();
    mbar_arrive_expect_tx(&bar, kResidRows * kFfn * 2);
    const uint64_t pol = policy_evict_first();
    for (int r = 0; r < kResidRows; ++r)
      bulk_g2s_stream(smem + static_cast<size_t>(r) * kFfn * 2, p.w + static_cast<size_t>(r0 + r) * kFfn, kFfn * 2,
                      &bar, pol);
  }
  const int orow = tid % kResidRows, oc = tid / kResidRows;  // owner of (row, clip) for the epilogue
  const bool owner = oc < C;
  const float bias = (p.b && owner) ? __half2float(p.b[r0 + orow]) : 0.f;
  __syncthreads();
  pdl_wait();
  pdl_trigger();
  const float hres = owner ? __half2float(p.h[static_cast<size_t>(oc) * kHidden + r0 + orow]) : 0.f;
  bool waited = false;
#pragma unroll 1
  for (int c0 = 0; c0 < C; c0 += 4) {
    float xf[4][2][8];
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        uint4 xv = make_uint4(0, 0, 0, 0);
        if (c0 + cc < C) xv = reinterpret_cast<const uint4*>(p.x + static_cast<size_t>(c0 + cc) * kFfn)[tid + 320 * j];
        const half2* px = reinterpret_cast<const half2*>(&xv);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __half22float2(px[e]);
          xf[cc][j][2 * e] = f.x;
          xf[cc][j][2 * e + 1] = f.y;
        }
      }
    }
    if (!waited) {
      if (!mbar_wait(&bar, 0)) flag_error(FW_DEVERR_TIMEOUT);
      waited = true;
    }
    float acc[32];  // rows 0-7 x clips 0-3, index 4 r + cc
    float tail[2][4];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = 0.f;
#pragma unroll
    for (int r = 0; r < kResidRows; ++r) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const uint4 wv = ws[r * kc + tid + 320 * j];
        const half2* pw = reinterpret_cast<const half2*>(&wv);
        float wf[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __half22float2(pw[e]);
          wf[2 * e] = f.x;
          wf[2 * e + 1] = f.y;
        }
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          float& a = r < 8 ? acc[4 * r + cc] : tail[r - 8][cc];
          if (j == 0) a = 0.f;
#pragma unroll
          for (int e = 0; e < 8; ++e) a = fmaf(wf[e], xf[cc][j][e], a);
        }
      }
    }
    const float s = warp_sum32_transpose(acc);  // lane l: row l / 4, clip c0 + l % 4
    if (c0 + (lane & 3) < C) red[warp][lane >> 2][c0 + (lane & 3)] = s;
#pragma unroll
    for (int rr = 0; rr < 2; ++rr)
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        const float t = warp_sum(tail[rr][cc]);
        if (lane == 0 && c0 + cc < C) red[warp][8 + rr][c0 + cc] = t;
      }
  }
  __syncthreads();
  if (owner) {
    float sum = 0.f;
#pragma unroll
    for (int w = 0; w < kBfc2Threads / 32; ++w) sum += red[w][orow][oc];
    p.h[static_cast<size_t>(oc) * kHidden + r0 + orow] = __float2half(hres + round_half(sum + bias));
  }
}

// ---------------------------------------------------------------------------------------------
// On-device decode loop (fw_decode_loop_*): the condition of a CUDA-graph WHILE node whose body is
// decode steps. It replaces the host loop of custom/model.py:208-215 (replay an 8-step graph, read the
// tokens back, stop at EOS or the token limit). ctrl (int64): [0] token limit, [1] EOS id,
// [2] stop at EOS (0/1), [3] body iterations run, [4] iteration cap. The loop continues while fewer
// than ctrl[0] tokens were generated, the last generated token is not EOS (when ctrl[2] is set) and
// the cap is not reached (a guard that makes the loop finite whatever the state holds).
__global__ void decode_loop_cond_kernel(const int64_t* __restrict__ state, const int64_t* __restrict__ tokens,
                                        int64_t* __restrict__ ctrl, cudaGraphConditionalHandle handle, int first,
                                        int window) {
  const int64_t it = first ? 0 : ctrl[3] + 1;
  ctrl[3] = it;
  const int64_t n = state[1];
  bool more = n < ctrl[0] && it < ctrl[4];
  // stop at EOS among the tokens the last iteration generated (its `window` steps)
  if (more && ctrl[2] != 0)
    for (int64_t i = n > window ? n - window : 0; i < n; ++i)
      if (tokens[i] == ctrl[1]) {
        more = false;
        break;
      }
  cudaGraphSetConditional(handle, more ? 1u : 0u);
}

// ---------------------------------------------------------------------------------------------
// Host launchers.
constexpr int kQkvRows = 24;   // 3840 / 24 = 160 CTAs
constexpr int kFc1Rows = 32;   // 5120 / 32 = 160 CTAs
constexpr int kSmallRows = 8;  // 1280 / 8 = 160 CTAs

static int rows_for(int n_out) {
  if (n_out >= 5120) return kFc1Rows;
  if (n_out >= 3840) return kQkvRows;
  return kSmallRows;
}

template <int kAct, int kRowsPerWarp>
static int launch_ln_gemv_t(const GemvParams& p, cudaStream_t s, bool pdl) {
  const int smem = p.rows_per_cta * kHidden * 2;
  auto kern = ln_gemv_kernel<kAct, kRowsPerWarp>;
  cudaError_t e = ensure_smem(kern, smem);
  if (e == cudaSuccess) {
    const int grid = (p.n_out + p.rows_per_cta - 1) / p.rows_per_cta;
    e = launch(kern, dim3(grid), dim3(256), smem, s, pdl, p);
  }
  return launch_status(e, "ln_gemv");
}

// fc1 of the decode step with the deferred residual of the cross block: 32 rows per CTA, clusters of
// kHeadCtas (the grid, 160 CTAs, is a multiple)
static int launch_ln_gemv_res(const GemvParams& p, cudaStream_t s) {
  const int smem = p.rows_per_cta * kHidden * 2;
  auto kern = ln_gemv_kernel<1, 4, true>;
  const int grid = (p.n_out + p.rows_per_cta - 1) / p.rows_per_cta;
  FW_REQUIRE(p.rows_per_cta == 32 && grid % kHeadCtas == 0, FW_ERR_SHAPE, "ln_gemv: deferred residual needs 32 rows per CTA");
  cudaError_t e = ensure_smem(kern, smem);
  if (e == cudaSuccess) e = launch_cluster(kern, dim3(grid), dim3(256), smem, s, true, kHeadCtas, p);
  return launch_status(e, "ln_gemv");
}

template <int kAct>
static int launch_ln_gemv(const GemvParams& p, cudaStream_t s, bool pdl) {
  switch (p.rows_per_cta) {
    case 8: return launch_ln_gemv_t<kAct, 1>(p, s, pdl);
    case 24: return launch_ln_gemv_t<kAct, 3>(p, s, pdl);
    case 32: return launch_ln_gemv_t<kAct, 4>(p, s, pdl);
    default: return set_error(FW_ERR_ARG, "ln_gemv: rows_per_cta must be 8, 24 or 32");
  }
}

template <int kChunks>
static int launch_gemv_residual_t(const GemvParams& p, cudaStream_t s, bool pdl) {
  auto kern = gemv_residual_kernel<kChunks>;
  const int smem = kResidRows * 256 * kChunks * 2;
  cudaError_t e = ensure_smem(kern, smem);
  if (e == cudaSuccess) {
    const int grid = (p.n_out + kResidRows - 1) / kResidRows;
    e = launch(kern, dim3(grid), dim3(kResidThreads), smem, s, pdl, p);
  }
  return launch_status(e, "gemv_residual");
}

static int launch_gemv_residual(const GemvParams& p, cudaStream_t s, bool pdl) {
  if (p.k == kHidden) return launch_gemv_residual_t<kHidden / 256>(p, s, pdl);
  if (p.k == kFfn) return launch_gemv_residual_t<kFfn / 256>(p, s, pdl);
  return set_error(FW_ERR_SHAPE, "gemv_residual: k must be %d or %d", kHidden, kFfn);
}

static int launch_attention(const AttnParams& p, int heads, int splits, cudaStream_t s, bool pdl) {
  cudaError_t e = launch(attn_split_kernel, dim3(heads, splits), dim3(64), 0, s, pdl, p);
  return launch_status(e, "decode_attention");
}

template <bool kSelf, bool kEmbed>
static int launch_head_block(const HeadBlockParams& p, int heads, cudaStream_t s, bool pdl) {
  auto kern = head_block_kernel<kSelf, kEmbed>;
  constexpr int smem = HeadBlockShape<kSelf>::kSmem;
  cudaError_t e = ensure_smem(kern, smem);
  if (e == cudaSuccess) e = launch_cluster(kern, dim3(kHeadCtas, heads), dim3(256), smem, s, pdl, kHeadCtas, p);
  return launch_status(e, kSelf ? "self_attention_block" : "cross_attention_block");
}

template <bool kLN, bool kFinalize>
static int launch_lm_head(LmParams p, cudaStream_t s, bool pdl) {
  auto kern = lm_head_kernel<kLN, kFinalize>;
  cudaError_t e = ensure_smem(kern, kLmSmem);
  if (e == cudaSuccess) {
    const int grid = num_sms();
    p.rows_per_cta = (p.vocab + grid - 1) / grid;
    if (p.rows_per_cta > kLmMaxRowsPerCta)
      return set_error(FW_ERR_SHAPE, "lm_head_argmax: vocab must be <= %d", kLmMaxRowsPerCta * grid);
    e = launch(kern, dim3(grid), dim3(256), kLmSmem, s, pdl, p);
  }
  return launch_status(e, "lm_head_argmax");
}

// 2-D uint8 tensor map over the int8 LM head [vocab][1280]: box 128 bytes x kQBoxRows rows, 128B
// swizzle; rows past the end read as zero.
static int make_lm_map(CUtensorMap* m, const void* wq, int vocab) {
  EncodeTiledFn enc = tensor_map_encode_fn();
  if (!enc) return set_error(FW_ERR_LAUNCH, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(kHidden), static_cast<cuuint64_t>(vocab)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(kHidden)};
  cuuint32_t box[2] = {kQChunk, kQBoxRows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(wq), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(FW_ERR_ARG, "tensor map encode failed (%d)", static_cast<int>(r));
  return FW_OK;
}

template <bool kLN, bool kFinalize, int kClips = 1>
static int launch_lm_head_q(LmParams p, cudaStream_t s, bool pdl) {
  auto kern = lm_head_q_kernel<kLN, kFinalize, kClips>;
  constexpr int smem = LmqShape<kClips>::kSmem;
  const int grid = num_sms();
  p.rows_per_cta = (p.vocab + grid - 1) / grid;
  if (p.rows_per_cta > kLmMaxRowsPerCta)
    return set_error(FW_ERR_SHAPE, "lm_head_argmax_q: vocab must be <= %d", kLmMaxRowsPerCta * grid);
  CUtensorMap map;
  int rc = make_lm_map(&map, p.wq, p.vocab);
  if (rc) return rc;
  cudaError_t e = ensure_smem(kern, smem);
  if (e == cudaSuccess) e = launch(kern, dim3(grid), dim3(256), smem, s, pdl, map, p);
  return launch_status(e, "lm_head_argmax_q");
}

template <int kAct, int kRowsPerWarp, bool kEmbed>
static int launch_bln_gemv(const BatchGemvParams& p, cudaStream_t s) {
  auto kern = bln_gemv_kernel<kAct, kRowsPerWarp, kEmbed>;
  using S = BlnShape<kRowsPerWarp>;
  cudaError_t e = ensure_smem(kern, S::kSmem);
  if (e == cudaSuccess)
    e = launch(kern, dim3((p.n_out + S::kRows - 1) / S::kRows), dim3(kBlnThreads), S::kSmem, s, true, p);
  return launch_status(e, "batch_ln_gemv");
}

static int launch_bout(const BatchOutParams& p, cudaStream_t s) {
  cudaError_t e = ensure_smem(bout_residual_kernel, kBoutSmem);
  if (e == cudaSuccess) e = launch(bout_residual_kernel, dim3(kHidden / kOutRowsB), dim3(kOutThreadsB), kBoutSmem, s, true, p);
  return launch_status(e, "batch_out_proj");
}

static int launch_bfc2(const BatchFc2Params& p, cudaStream_t s) {
  constexpr int smem = kResidRows * kFfn * 2;
  cudaError_t e = ensure_smem(bfc2_residual_kernel, smem);
  if (e == cudaSuccess) e = launch(bfc2_residual_kernel, dim3(kHidden / kResidRows), dim3(kBfc2Threads), smem, s, true, p);
  return launch_status(e, "batch_fc2");
}

// ---------------------------------------------------------------------------------------------
// Split-K attention without caller-allocated workspace (fw_decode_attention_noalloc).
// The fp32 split partials live in this fixed device array instead: per GPU that loads the library,
// kNoAllocMaxSlots head-splits x (64 accumulators + max + sum) x 4 bytes = 528 KB, held until the
// process exits. Host code must not hand the symbol itself to a kernel (on the host it only names
// a stand-in); its device address is looked up once per device with cudaGetSymbolAddress.
constexpr int kNoAllocMaxSlots = 2048;  // heads * ceil(max_len / 64)
static __device__ __align__(256) float g_attn_noalloc_scratch[kNoAllocMaxSlots * (kHeadDim + 2)];

// Device address of g_attn_noalloc_scratch in the current device's current context. The address is
// looked up on the first call per device and cached together with the context it belongs to; a call
// made in another context of that device (after cudaDeviceReset, or a primary context that was
// released and re-created) looks it up again, since a new context loads the module afresh. Returns
// nullptr and sets the error message on failure.
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

static CUcontext current_context() {
  static CtxGetCurrentFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  }
  CUcontext ctx = nullptr;
  if (fn != nullptr && fn(&ctx) != CUDA_SUCCESS) ctx = nullptr;
  return ctx;
}

static float* noalloc_scratch() {
  static std::mutex mu;
  static float* cached[64] = {nullptr};
  static CUcontext cached_ctx[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_error(FW_ERR_LAUNCH, "decode_attention_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    return nullptr;
  }
  if (dev < 0 || dev >= 64) {
    set_error(FW_ERR_UNSUPPORTED, "decode_attention_noalloc: device index %d out of range", dev);
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  const CUcontext ctx = current_context();
  if (cached[dev] == nullptr || ctx == nullptr || ctx != cached_ctx[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error(FW_ERR_LAUNCH, "decode_attention_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      return nullptr;
    }
    cached[dev] = static_cast<float*>(p);
    cached_ctx[dev] = current_context();  // the lookup made the device's primary context current
  }
  return cached[dev];
}

unsigned int read_decode_errors(bool clear) {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_fw_dev_error, sizeof(v));
  if (clear) {
    const unsigned int zero = 0;
    cudaMemcpyToSymbol(g_fw_dev_error, &zero, sizeof(zero));
  }
  return v;
}

}  // namespace fw

using namespace fw;

extern "C" {

int fw_add_layernorm(void* h, const void* x, const void* gamma, const void* beta, void* y, int hidden, float eps,
                     fw_stream_t stream) {
  FW_REQUIRE(h && gamma && beta && y, FW_ERR_NULL, "add_layernorm: h, gamma, beta and y are required");
  FW_REQUIRE(hidden == kHidden, FW_ERR_SHAPE, "hidden size must be %d", kHidden);
  cudaError_t e = launch(add_layernorm_kernel, dim3(1), dim3(256), 0, static_cast<cudaStream_t>(stream), false,
                         static_cast<half*>(h), static_cast<const half*>(x), static_cast<const half*>(gamma),
                         static_cast<const half*>(beta), static_cast<half*>(y), eps);
  return launch_status(e, "add_layernorm");
}

int fw_decode_attention(const void* q, void* k, void* v, void* out, const int64_t* len_state, const void* k_new,
                        const void* v_new, float* part_m, int64_t part_m_numel, float* part_l, int64_t part_l_numel,
                        float* part_acc, int64_t part_acc_numel, int heads, int max_len, float scale,
                        fw_stream_t stream) {
  FW_REQUIRE(q && k && v && out && part_m && part_l && part_acc, FW_ERR_NULL,
             "decode_attention: q, k, v, out and the workspace are required");
  FW_REQUIRE((k_new != nullptr) == (v_new != nullptr) && (k_new != nullptr) == (len_state != nullptr), FW_ERR_ARG,
             "len_state, k_new and v_new must be given together");
  FW_REQUIRE(heads > 0 && max_len > 0, FW_ERR_SHAPE, "k, v must be [heads, max_len, 64]");
  FW_REQUIRE(max_len <= kMaxSplits * kSplitKeys, FW_ERR_SHAPE, "decode_attention: max_len must be <= %d",
             kMaxSplits * kSplitKeys);
  const int splits = (max_len + kSplitKeys - 1) / kSplitKeys;
  FW_REQUIRE(part_m_numel >= int64_t(heads) * splits && part_l_numel >= int64_t(heads) * splits &&
                 part_acc_numel >= int64_t(heads) * splits * kHeadDim,
             FW_ERR_SHAPE, "workspace too small for %d splits", splits);
  FW_REQUIRE(aligned16(k) && aligned16(v), FW_ERR_ALIGN, "k and v must be 16-byte aligned");
  AttnParams p{static_cast<const half*>(q), static_cast<half*>(k), static_cast<half*>(v),
               static_cast<const half*>(k_new), static_cast<const half*>(v_new), len_state, max_len, scale,
               part_m, part_l, part_acc, static_cast<half*>(out), nullptr};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = launch_attention(p, heads, splits, s, false);
  if (rc) return rc;
  cudaError_t e = launch(attn_combine_kernel, dim3(heads), dim3(kHeadDim), 0, s, false,
                         static_cast<const float*>(part_m), static_cast<const float*>(part_l),
                         static_cast<const float*>(part_acc), static_cast<half*>(out), splits);
  return launch_status(e, "decode_attention_combine");
}

int fw_decode_attention_noalloc(const void* q, void* k, void* v, void* out, const int64_t* len_state,
                                const void* k_new, const void* v_new, int heads, int max_len, float scale,
                                fw_stream_t stream) {
  FW_REQUIRE(q && k && v && out, FW_ERR_NULL, "decode_attention_noalloc: q, k, v and out are required");
  FW_REQUIRE((k_new != nullptr) == (v_new != nullptr) && (k_new != nullptr) == (len_state != nullptr), FW_ERR_ARG,
             "len_state, k_new and v_new must be given together");
  FW_REQUIRE(heads > 0 && max_len > 0, FW_ERR_SHAPE, "k, v must be [heads, max_len, 64]");
  FW_REQUIRE(max_len <= kMaxSplits * kSplitKeys, FW_ERR_SHAPE, "decode_attention_noalloc: max_len must be <= %d",
             kMaxSplits * kSplitKeys);
  const int splits = (max_len + kSplitKeys - 1) / kSplitKeys;
  FW_REQUIRE(int64_t(heads) * splits <= kNoAllocMaxSlots, FW_ERR_SHAPE,
             "decode_attention_noalloc: heads * ceil(max_len / 64) = %lld exceeds the fixed scratch of %d "
             "head-splits; use fw_decode_attention with a caller workspace",
             static_cast<long long>(int64_t(heads) * splits), kNoAllocMaxSlots);
  FW_REQUIRE(aligned16(k) && aligned16(v), FW_ERR_ALIGN, "k and v must be 16-byte aligned");
  float* scratch = noalloc_scratch();
  if (scratch == nullptr) return FW_ERR_LAUNCH;
  float* part_acc = scratch;
  float* part_m = scratch + kNoAllocMaxSlots * kHeadDim;
  float* part_l = part_m + kNoAllocMaxSlots;
  AttnParams p{static_cast<const half*>(q), static_cast<half*>(k), static_cast<half*>(v),
               static_cast<const half*>(k_new), static_cast<const half*>(v_new), len_state, max_len, scale,
               part_m, part_l, part_acc, static_cast<half*>(out), nullptr};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = launch_attention(p, heads, splits, s, false);
  if (rc) return rc;
  cudaError_t e = launch(attn_combine_kernel, dim3(heads), dim3(kHeadDim), 0, s, false,
                         static_cast<const float*>(part_m), static_cast<const float*>(part_l),
                         static_cast<const float*>(part_acc), static_cast<half*>(out), splits);
  return launch_status(e, "decode_attention_noalloc_combine");
}

int fw_lm_head_argmax(const void* h, const void* w, const bool* suppress, int vocab, int hidden, int64_t* best,
                      fw_stream_t stream) {
  FW_REQUIRE(h && w && suppress && best, FW_ERR_NULL, "lm_head_argmax: h, w, suppress and best are required");
  FW_REQUIRE(hidden == kHidden, FW_ERR_SHAPE, "hidden size must be %d", kHidden);
  FW_REQUIRE(vocab > 0, FW_ERR_SHAPE, "suppress must be bool [vocab]");
  FW_REQUIRE(aligned16(h) && aligned16(w), FW_ERR_ALIGN, "h and w must be 16-byte aligned");
  LmParams p{};
  p.h = static_cast<const half*>(h);
  p.w = static_cast<const half*>(w);
  p.vocab = vocab;
  p.mask = suppress;
  p.best = reinterpret_cast<unsigned long long*>(best);
  return launch_lm_head<false, false>(p, static_cast<cudaStream_t>(stream), false);
}

int fw_lm_quantize(const void* w, int vocab, int hidden, void* wq, void* rp, fw_stream_t stream) {
  FW_REQUIRE(w && wq && rp, FW_ERR_NULL, "lm_quantize: w, wq and rp are required");
  FW_REQUIRE(hidden == kHidden, FW_ERR_SHAPE, "hidden size must be %d", kHidden);
  FW_REQUIRE(vocab > 0, FW_ERR_SHAPE, "lm_quantize: vocab must be positive");
  FW_REQUIRE(aligned16(w) && aligned16(wq) && aligned16(rp), FW_ERR_ALIGN, "w, wq and rp must be 16-byte aligned");
  cudaError_t e = launch(lm_quantize_kernel, dim3((vocab + 7) / 8), dim3(256), 0, static_cast<cudaStream_t>(stream),
                         false, static_cast<const half*>(w), vocab, static_cast<int8_t*>(wq), static_cast<float4*>(rp));
  return launch_status(e, "lm_quantize");
}

int fw_lm_head_argmax_q(const void* h, const void* w, const void* wq, const void* rp, const bool* suppress, int vocab,
                        int hidden, int64_t* best, fw_stream_t stream) {
  FW_REQUIRE(h && w && wq && rp && suppress && best, FW_ERR_NULL,
             "lm_head_argmax_q: h, w, wq, rp, suppress and best are required");
  FW_REQUIRE(hidden == kHidden, FW_ERR_SHAPE, "hidden size must be %d", kHidden);
  FW_REQUIRE(vocab > 0, FW_ERR_SHAPE, "suppress must be bool [vocab]");
  FW_REQUIRE(aligned16(h) && aligned16(w) && aligned16(wq) && aligned16(rp), FW_ERR_ALIGN,
             "h, w, wq and rp must be 16-byte aligned");
  LmParams p{};
  p.h = static_cast<const half*>(h);
  p.w = static_cast<const half*>(w);
  p.wq = static_cast<const int8_t*>(wq);
  p.rp = static_cast<const float4*>(rp);
  p.vocab = vocab;
  p.mask = suppress;
  p.best = reinterpret_cast<unsigned long long*>(best);
  return launch_lm_head_q<false, false>(p, static_cast<cudaStream_t>(stream), false);
}

int fw_argmax_finalize(int64_t* best, int64_t* tokens, int64_t n_tokens, int64_t* state, int64_t* cur, int max_pos,
                       fw_stream_t stream) {
  FW_REQUIRE(best && tokens && state && cur, FW_ERR_NULL, "argmax_finalize: best, tokens, state and cur are required");
  FW_REQUIRE(max_pos > 0 && n_tokens >= 0, FW_ERR_SHAPE, "max_pos must be positive");
  cudaError_t e = launch(argmax_finalize_kernel, dim3(1), dim3(1), 0, static_cast<cudaStream_t>(stream), false,
                         reinterpret_cast<unsigned long long*>(best), tokens, n_tokens, state, cur, max_pos);
  return launch_status(e, "argmax_finalize");
}

int fw_embed_pos(const void* embed, const void* pos_embed, const int64_t* ids, const int64_t* positions, void* out,
                 int n, int vocab, int max_pos, int hidden, fw_stream_t stream) {
  FW_REQUIRE(embed && pos_embed && ids && positions && out, FW_ERR_NULL, "embed_pos: all pointers are required");
  FW_REQUIRE(n >= 0 && vocab > 0 && max_pos > 0 && hidden > 0 && hidden % 2 == 0, FW_ERR_SHAPE,
             "embed_pos: bad sizes");
  if (n == 0) return FW_OK;
  cudaError_t e = launch(embed_pos_kernel, dim3(n), dim3(256), 0, static_cast<cudaStream_t>(stream), false,
                         static_cast<const half*>(embed), static_cast<const half*>(pos_embed), ids, positions,
                         static_cast<half*>(out), n, vocab, max_pos, hidden);
  return launch_status(e, "embed_pos");
}

int fw_gelu(const void* x, void* y, int64_t n, fw_stream_t stream) {
  FW_REQUIRE(x && y, FW_ERR_NULL, "gelu: x and y are required");
  FW_REQUIRE(n >= 0, FW_ERR_SHAPE, "gelu: n must be >= 0");
  if (n == 0) return FW_OK;
  const int64_t blocks = (n + 255) / 256;
  const int grid = static_cast<int>(blocks < 4096 ? blocks : 4096);
  cudaError_t e = launch(gelu_kernel, dim3(grid), dim3(256), 0, static_cast<cudaStream_t>(stream), false,
                         static_cast<const half*>(x), static_cast<half*>(y), n);
  return launch_status(e, "gelu");
}

int fw_argmax_f16(const void* logits, int64_t n, const bool* suppress, int64_t* key, int64_t* out_index,
                  fw_stream_t stream) {
  FW_REQUIRE(logits && key && out_index, FW_ERR_NULL, "argmax_f16: logits, key and out_index are required");
  FW_REQUIRE(n > 0 && n < (int64_t(1) << 31), FW_ERR_SHAPE, "argmax_f16: n out of range");
  FW_REQUIRE(aligned16(logits), FW_ERR_ALIGN, "argmax_f16: logits must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t chunks = (n / 8 + 255) / 256;
  int grid = static_cast<int>(chunks < 2 * num_sms() ? chunks : 2 * num_sms());
  if (grid < 1) grid = 1;
  cudaError_t e = launch(argmax_f16_kernel, dim3(grid), dim3(256), 0, s, false, static_cast<const half*>(logits), n,
                         suppress, reinterpret_cast<unsigned long long*>(key));
  int rc = launch_status(e, "argmax_f16");
  if (rc) return rc;
  e = launch(argmax_index_kernel, dim3(1), dim3(1), 0, s, false, reinterpret_cast<unsigned long long*>(key),
             out_index);
  return launch_status(e, "argmax_index");
}

int fw_ln_gemv(const void* h, const void* gamma, const void* beta, float eps, const void* w, const void* b, void* out,
               int n_out, int hidden, int act, fw_stream_t stream) {
  FW_REQUIRE(h && gamma && beta && w && out, FW_ERR_NULL, "ln_gemv: h, gamma, beta, w and out are required");
  FW_REQUIRE(hidden == kHidden, FW_ERR_SHAPE, "hidden size must be %d", kHidden);
  FW_REQUIRE(n_out > 0, FW_ERR_SHAPE, "ln_gemv: n_out must be positive");
  FW_REQUIRE(act == 0 || act == 1, FW_ERR_ARG, "ln_gemv: act must be 0 (none) or 1 (gelu)");
  FW_REQUIRE(aligned16(w), FW_ERR_ALIGN, "ln_gemv: w must be 16-byte aligned");
  GemvParams p{};
  p.w = static_cast<const half*>(w);
  p.b = static_cast<const half*>(b);
  p.out = static_cast<half*>(out);
  p.n_out = n_out;
  p.k = kHidden;
  p.rows_per_cta = rows_for(n_out);
  p.h = static_cast<const half*>(h);
  p.gamma = static_cast<const half*>(gamma);
  p.beta = static_cast<const half*>(beta);
  p.eps = eps;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return act ? launch_ln_gemv<1>(p, s, false) : launch_ln_gemv<0>(p, s, false);
}

int fw_gemv_residual(const void* x, int k, const void* w, const void* b, void* h, int n_out, fw_stream_t stream) {
  FW_REQUIRE(x && w && h, FW_ERR_NULL, "gemv_residual: x, w and h are required");
  FW_REQUIRE(k == kHidden || k == kFfn, FW_ERR_SHAPE, "gemv_residual: k must be %d or %d", kHidden, kFfn);
  FW_REQUIRE(n_out > 0, FW_ERR_SHAPE, "gemv_residual: n_out must be positive");
  FW_REQUIRE(aligned16(w) && aligned16(x), FW_ERR_ALIGN, "gemv_residual: w and x must be 16-byte aligned");
  GemvParams p{};
  p.w = static_cast<const half*>(w);
  p.b = static_cast<const half*>(b);
  p.n_out = n_out;
  p.k = k;
  p.rows_per_cta = kResidRows;
  p.x = static_cast<const half*>(x);
  p.h_res = static_cast<half*>(h);
  return launch_gemv_residual(p, static_cast<cudaStream_t>(stream), false);
}

}  // extern "C"

namespace fw {

// Checks a decoder descriptor (shared by fw_decoder_step and fw_decoder_step_trace).
static int check_decoder(const fw_decoder_t* d) {
  FW_REQUIRE(d != nullptr, FW_ERR_NULL, "decoder_step: descriptor is NULL");
  FW_REQUIRE(d->n_layers > 0 && d->n_layers <= FW_MAX_LAYERS, FW_ERR_SHAPE, "decoder_step: bad layer count");
  FW_REQUIRE(d->heads * kHeadDim == kHidden, FW_ERR_SHAPE, "decoder_step: heads * 64 must be %d", kHidden);
  FW_REQUIRE(d->max_pos > 0 && d->enc_len > 0 && d->vocab > 0, FW_ERR_SHAPE, "decoder_step: bad sizes");
  FW_REQUIRE(d->embed && d->pos_embed && d->lm_head && d->final_g && d->final_b && d->h && d->cq && d->ffn &&
                 d->part_acc && d->counters && d->cur && d->state && d->tokens && d->best,
             FW_ERR_NULL, "decoder_step: a required pointer is NULL");
  FW_REQUIRE(aligned16(d->h) && aligned16(d->cq), FW_ERR_ALIGN, "decoder_step: h and cq must be 16-byte aligned");
  FW_REQUIRE(d->prompt_len == 0 || d->prompt != nullptr, FW_ERR_NULL, "decoder_step: prompt is NULL");
  FW_REQUIRE((d->lm_q == nullptr) == (d->lm_rp == nullptr), FW_ERR_NULL, "decoder_step: set both lm_q and lm_rp or neither");
  FW_REQUIRE(d->lm_q == nullptr || (aligned16(d->lm_q) && aligned16(d->lm_rp)), FW_ERR_ALIGN,
             "decoder_step: lm_q and lm_rp must be 16-byte aligned");
  const int self_splits = (d->max_pos + kSplitKeys - 1) / kSplitKeys;
  const int cross_splits = (d->enc_len + kSplitKeys - 1) / kSplitKeys;
  FW_REQUIRE(self_splits <= kHeadCtas && cross_splits <= kHeadCtas * kHeadMaxUnits, FW_ERR_SHAPE,
             "decoder_step: max_pos must be <= %d and enc_len <= %d", kHeadCtas * kSplitKeys,
             kHeadCtas * kHeadMaxUnits * kSplitKeys);
  FW_REQUIRE(d->ws_splits * kHeadDim >= 2 * kHidden, FW_ERR_SHAPE,
             "decoder_step: part_acc must hold 2 * heads * 1280 floats (ws_splits >= %d)", 2 * kHidden / kHeadDim);
  return FW_OK;
}

// Launch `block` of layer `l` of the decode step: 0 self-attention block, 1 cross-attention block,
// 2 LN3 + fc1 + GELU, 3 fc2 + residual; block 4 (l ignored) is the LM head with the final LayerNorm,
// argmax and token bookkeeping. `tl` (this layer's trace record) and `y_out` are optional outputs of
// fw_decoder_step_trace.
static int decoder_launch(const fw_decoder_t* d, int l, int block, cudaStream_t s, half* tl, half* y_out) {
  half* h = static_cast<half*>(d->h);
  half* ffn = static_cast<half*>(d->ffn);
  if (block == 4) {
    LmParams m{};
    m.h = h;
    m.gamma = static_cast<const half*>(d->final_g);
    m.beta = static_cast<const half*>(d->final_b);
    m.eps = d->eps;
    m.w = static_cast<const half*>(d->lm_head);
    m.vocab = d->vocab;
    m.mask = d->base_mask;
    m.first_mask = d->first_mask;
    m.best = reinterpret_cast<unsigned long long*>(d->best);
    m.counter = d->counters + d->heads;
    m.tokens = d->tokens;
    m.n_tokens = d->n_tokens;
    m.state = d->state;
    m.cur = d->cur;
    m.max_pos = d->max_pos;
    m.prompt_len = d->prompt_len;
    m.y_out = y_out;
    if (d->lm_q != nullptr) {
      m.wq = static_cast<const int8_t*>(d->lm_q);
      m.rp = static_cast<const float4*>(d->lm_rp);
      return launch_lm_head_q<true, true>(m, s, true);
    }
    return launch_lm_head<true, true>(m, s, true);
  }
  const fw_decoder_layer_t& L = d->layers[l];
  if (block == 0) {
    // LN1 + q/k/v (+ embedding on layer 0) + self attention with the cache write + out_proj + residual
    HeadBlockParams a{};
    a.h = h;
    a.gamma = static_cast<const half*>(L.ln1_g);
    a.beta = static_cast<const half*>(L.ln1_b);
    a.eps = d->eps;
    a.embed = static_cast<const half*>(d->embed);
    a.pos_embed = static_cast<const half*>(d->pos_embed);
    a.cur = d->cur;
    a.prompt = d->prompt;
    a.prompt_len = d->prompt_len;
    a.vocab = d->vocab;
    a.state = d->state;
    a.max_pos = d->max_pos;
    a.state_early = l > 0;  // on layer 0 the previous launch (LM head) advances the position
    a.w = static_cast<const half*>(L.qkv_w);
    a.b = static_cast<const half*>(L.qkv_b);
    a.k = static_cast<half*>(L.self_k);
    a.v = static_cast<half*>(L.self_v);
    a.kv_len = d->max_pos;
    a.scale = d->scale;
    a.wo = static_cast<const half*>(L.out_w);
    a.part = d->part_acc;  // left for the cross block, which forms h + this block's output itself
    a.attn_out = tl ? tl + FW_TRACE_SELF_ATTN : static_cast<half*>(d->attn);
    return l == 0 ? launch_head_block<true, true>(a, d->heads, s, true)
                  : launch_head_block<true, false>(a, d->heads, s, true);
  }
  if (block == 1) {
    // LN2 + cross q + cross attention + cross out_proj + residual
    HeadBlockParams c{};
    c.h = h;
    c.gamma = static_cast<const half*>(L.ln2_g);
    c.beta = static_cast<const half*>(L.ln2_b);
    c.eps = d->eps;
    c.state = d->state;
    c.max_pos = d->max_pos;
    c.w = static_cast<const half*>(L.cq_w);
    c.b = static_cast<const half*>(L.cq_b);
    c.k = const_cast<half*>(static_cast<const half*>(L.cross_k));
    c.v = const_cast<half*>(static_cast<const half*>(L.cross_v));
    c.kv_len = d->enc_len;
    c.scale = d->scale;
    c.wo = static_cast<const half*>(L.co_w);  // (its bias co_b is added by fc1)
    c.res_part = d->part_acc;  // the self block's partials, summed here into h + its output
    c.res_bias = static_cast<const half*>(L.out_b);
    c.h_in_out = static_cast<half*>(d->cq);  // that residual, for fc1
    c.part = d->part_acc + static_cast<size_t>(d->heads) * kHidden;  // left for fc1
    c.attn_out = tl ? tl + FW_TRACE_CROSS_ATTN : nullptr;
    return launch_head_block<false, false>(c, d->heads, s, true);
  }
  if (block == 2) {
    // LN3 + fc1 + GELU
    GemvParams g{};
    g.w = static_cast<const half*>(L.fc1_w);
    g.b = static_cast<const half*>(L.fc1_b);
    g.out = ffn;
    g.n_out = kFfn;
    g.k = kHidden;
    g.rows_per_cta = kFc1Rows;
    g.h = static_cast<const half*>(d->cq);  // the residual after the self block, + the cross partials:
    g.res_part = d->part_acc + static_cast<size_t>(d->heads) * kHidden;
    g.res_bias = static_cast<const half*>(L.co_b);
    g.h_out = h;  // the residual after the cross block, fc2's residual input
    g.gamma = static_cast<const half*>(L.ln3_g);
    g.beta = static_cast<const half*>(L.ln3_b);
    g.eps = d->eps;
    return launch_ln_gemv_res(g, s);
  }
  // fc2 + residual
  GemvParams r{};
  r.w = static_cast<const half*>(L.fc2_w);
  r.b = static_cast<const half*>(L.fc2_b);
  r.n_out = kHidden;
  r.k = kFfn;
  r.rows_per_cta = kResidRows;
  r.x = ffn;
  r.h_res = h;
  return launch_gemv_residual(r, s, true);
}

// One decode step: 4 launches per layer and the LM head. With `trace` set (fw_decoder_step_trace),
// the same launches also leave each block's output in `trace` (FW_TRACE_* layout): the attention
// outputs and the final LayerNorm row are written by the kernels themselves, the residual stream and
// the fc1 output are copied after the launch that produced them.
static int decoder_one_step(const fw_decoder_t* d, cudaStream_t s, half* trace) {
  half* h = static_cast<half*>(d->h);
  auto snap = [&](half* dst, const void* src, int n) -> int {
    cudaError_t e = cudaMemcpyAsync(dst, src, static_cast<size_t>(n) * sizeof(half), cudaMemcpyDeviceToDevice, s);
    return e == cudaSuccess ? FW_OK : set_error(FW_ERR_LAUNCH, "decoder_step_trace: copy: %s", cudaGetErrorString(e));
  };
  // after the cross block: the residual after the self block (formed by the cross block, in cq); after
  // fc1: the residual after the cross block (formed by fc1, in h) and the fc1 output; after fc2: h
  const half* cq = static_cast<const half*>(d->cq);
  for (int l = 0; l < d->n_layers; ++l) {
    half* tl = trace ? trace + static_cast<size_t>(l) * FW_TRACE_LAYER : nullptr;
    for (int block = 0; block < 4; ++block) {
      int rc = decoder_launch(d, l, block, s, tl, nullptr);
      if (rc) return rc;
      if (tl && block == 1 && (rc = snap(tl + FW_TRACE_H_SELF, cq, kHidden))) return rc;
      if (tl && block == 2 && ((rc = snap(tl + FW_TRACE_H_CROSS, h, kHidden)) || (rc = snap(tl + FW_TRACE_FFN, d->ffn, kFfn))))
        return rc;
      if (tl && block == 3 && (rc = snap(tl + FW_TRACE_H_FFN, h, kHidden))) return rc;
    }
  }
  return decoder_launch(d, 0, 4, s, nullptr,
                        trace ? trace + static_cast<size_t>(d->n_layers) * FW_TRACE_LAYER : nullptr);
}

}  // namespace fw

extern "C" {

int fw_decoder_step(const fw_decoder_t* d, int steps, fw_stream_t stream) {
  int rc = check_decoder(d);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int step = 0; step < steps; ++step)
    if ((rc = decoder_one_step(d, s, nullptr))) return rc;
  return FW_OK;
}

int fw_decoder_launch(const fw_decoder_t* d, int layer, int block, fw_stream_t stream) {
  int rc = check_decoder(d);
  if (rc) return rc;
  FW_REQUIRE(block >= 0 && block <= 4, FW_ERR_ARG, "decoder_launch: block must be 0..4");
  FW_REQUIRE(block == 4 || (layer >= 0 && layer < d->n_layers), FW_ERR_ARG, "decoder_launch: layer out of range");
  return decoder_launch(d, block == 4 ? 0 : layer, block, static_cast<cudaStream_t>(stream), nullptr, nullptr);
}

int fw_decoder_step_trace(const fw_decoder_t* d, void* trace, fw_stream_t stream) {
  int rc = check_decoder(d);
  if (rc) return rc;
  FW_REQUIRE(trace != nullptr, FW_ERR_NULL, "decoder_step_trace: trace is NULL");
  FW_REQUIRE(aligned16(trace), FW_ERR_ALIGN, "decoder_step_trace: trace must be 16-byte aligned");
  return decoder_one_step(d, static_cast<cudaStream_t>(stream), static_cast<half*>(trace));
}

}  // extern "C"

namespace fw {

// Checks a batched decoder descriptor (fw_batch_decoder_step, fw_batch_decoder_launch).
static int check_batch_decoder(const fw_batch_decoder_t* d) {
  FW_REQUIRE(d != nullptr, FW_ERR_NULL, "batch_decoder_step: descriptor is NULL");
  FW_REQUIRE(d->clips > 0 && d->clips <= kMaxClips, FW_ERR_SHAPE, "batch_decoder_step: clips must be 1..%d",
             kMaxClips);
  FW_REQUIRE(d->n_layers > 0 && d->n_layers <= FW_MAX_LAYERS, FW_ERR_SHAPE, "batch_decoder_step: bad layer count");
  FW_REQUIRE(d->heads * kHeadDim == kHidden, FW_ERR_SHAPE, "batch_decoder_step: heads * 64 must be %d", kHidden);
  FW_REQUIRE(d->max_pos > 0 && d->enc_len > 0 && d->vocab > 0 && d->n_tokens > 0, FW_ERR_SHAPE,
             "batch_decoder_step: bad sizes");
  FW_REQUIRE(d->max_pos <= kMaxSplits * kSplitKeys && d->enc_len <= kMaxSplits * kSplitKeys, FW_ERR_SHAPE,
             "batch_decoder_step: max_pos and enc_len must be <= %d", kMaxSplits * kSplitKeys);
  FW_REQUIRE(d->embed && d->pos_embed && d->lm_head && d->final_g && d->final_b && d->h && d->qkv && d->attn &&
                 d->ffn && d->part_m && d->part_l && d->part_acc && d->counters && d->cur && d->state && d->tokens &&
                 d->best && d->lm_q && d->lm_rp,
             FW_ERR_NULL, "batch_decoder_step: a required pointer is NULL");
  FW_REQUIRE(d->prompt_len == 0 || d->prompt != nullptr, FW_ERR_NULL, "batch_decoder_step: prompt is NULL");
  const int self_splits = (d->max_pos + kSplitKeys - 1) / kSplitKeys;
  const int cross_splits = (d->enc_len + kSplitKeys - 1) / kSplitKeys;
  FW_REQUIRE(d->ws_splits >= self_splits && d->ws_splits >= cross_splits, FW_ERR_SHAPE,
             "batch_decoder_step: ws_splits must be >= %d", self_splits > cross_splits ? self_splits : cross_splits);
  FW_REQUIRE(d->self_clip_stride % 8 == 0 && d->cross_clip_stride % 8 == 0 && aligned16(d->lm_q) &&
                 aligned16(d->lm_rp) && aligned16(d->h) && aligned16(d->qkv) && aligned16(d->attn) && aligned16(d->ffn),
             FW_ERR_ALIGN, "batch_decoder_step: buffers and clip strides must be 16-byte aligned");
  for (int l = 0; l < d->n_layers; ++l) {
    const fw_decoder_layer_t& L = d->layers[l];
    FW_REQUIRE(L.self_k && L.self_v && L.cross_k && L.cross_v && L.qkv_w && L.out_w && L.cq_w && L.co_w && L.fc1_w &&
                   L.fc2_w && L.ln1_g && L.ln1_b && L.ln2_g && L.ln2_b && L.ln3_g && L.ln3_b,
               FW_ERR_NULL, "batch_decoder_step: layer %d is missing a weight or cache pointer", l);
    FW_REQUIRE(aligned16(L.self_k) && aligned16(L.self_v) && aligned16(L.cross_k) && aligned16(L.cross_v),
               FW_ERR_ALIGN, "batch_decoder_step: caches must be 16-byte aligned");
  }
  return FW_OK;
}

// Launch `block` of layer `l` of the batched step: 0 LN1 + q/k/v (layer 0: embedding), 1 self
// attention, 2 out_proj + residual, 3 LN2 + cross q, 4 cross attention, 5 cross out_proj + residual,
// 6 LN3 + fc1 + GELU, 7 fc2 + residual; block 8 (l ignored) is the LM head of all clips.
static int batch_launch(const fw_batch_decoder_t* d, int l, int block, cudaStream_t s) {
  const int C = d->clips;
  half* h = static_cast<half*>(d->h);
  half* qkv = static_cast<half*>(d->qkv);
  half* attn = static_cast<half*>(d->attn);
  half* ffn = static_cast<half*>(d->ffn);
  if (block == 8) {
    LmParams m{};
    m.h = h;
    m.gamma = static_cast<const half*>(d->final_g);
    m.beta = static_cast<const half*>(d->final_b);
    m.eps = d->eps;
    m.w = static_cast<const half*>(d->lm_head);
    m.wq = static_cast<const int8_t*>(d->lm_q);
    m.rp = static_cast<const float4*>(d->lm_rp);
    m.vocab = d->vocab;
    m.mask = d->base_mask;
    m.first_mask = d->first_mask;
    m.best = reinterpret_cast<unsigned long long*>(d->best);
    m.counter = d->counters + C * d->heads;
    m.tokens = d->tokens;
    m.n_tokens = d->n_tokens;
    m.tokens_stride = d->n_tokens;
    m.state = d->state;
    m.cur = d->cur;
    m.max_pos = d->max_pos;
    m.prompt_len = d->prompt_len;
    m.clips = C;
    return launch_lm_head_q<true, true, kMaxClips>(m, s, true);
  }
  const fw_decoder_layer_t& L = d->layers[l];
  BatchGemvParams g{};
  g.clips = C;
  g.h = h;
  g.eps = d->eps;
  g.out = qkv;
  g.out_stride = 3 * kHidden;
  if (block == 0) {  // LN1 + q/k/v (layer 0: h from the token embedding and position)
    g.w = static_cast<const half*>(L.qkv_w);
    g.b = static_cast<const half*>(L.qkv_b);
    g.n_out = 3 * kHidden;
    g.gamma = static_cast<const half*>(L.ln1_g);
    g.beta = static_cast<const half*>(L.ln1_b);
    g.embed = static_cast<const half*>(d->embed);
    g.pos_embed = static_cast<const half*>(d->pos_embed);
    g.cur = d->cur;
    g.state = d->state;
    g.prompt = d->prompt;
    g.prompt_len = d->prompt_len;
    g.vocab = d->vocab;
    g.max_pos = d->max_pos;
    g.h_out = h;
    return l == 0 ? launch_bln_gemv<0, 4, true>(g, s) : launch_bln_gemv<0, 4, false>(g, s);
  }
  if (block == 1 || block == 4) {  // self attention (cache write, fused combine) / cross attention
    const bool self = block == 1;
    AttnParams a{};
    a.q = qkv;
    a.k = const_cast<half*>(static_cast<const half*>(self ? L.self_k : L.cross_k));
    a.v = const_cast<half*>(static_cast<const half*>(self ? L.self_v : L.cross_v));
    if (self) {
      a.k_new = qkv + kHidden;
      a.v_new = qkv + 2 * kHidden;
      a.len_state = d->state;
      a.clip_new = 3 * kHidden;
      a.clip_state = 2;
    }
    a.max_len = self ? d->max_pos : d->enc_len;
    a.scale = d->scale;
    a.part_m = d->part_m;
    a.part_l = d->part_l;
    a.part_acc = d->part_acc;
    a.out = attn;
    a.counters = d->counters;
    a.clip_q = 3 * kHidden;
    a.clip_kv = self ? d->self_clip_stride : d->cross_clip_stride;
    a.clip_out = kHidden;
    const int splits = (a.max_len + kSplitKeys - 1) / kSplitKeys;
    cudaError_t e = launch(attn_split_kernel, dim3(d->heads, splits, C), dim3(64), 0, s, true, a);
    return launch_status(e, self ? "batch_self_attention" : "batch_cross_attention");
  }
  if (block == 2 || block == 5) {  // (cross) out_proj + residual
    BatchOutParams o{static_cast<const half*>(block == 2 ? L.out_w : L.co_w),
                     static_cast<const half*>(block == 2 ? L.out_b : L.co_b), attn, h, C};
    return launch_bout(o, s);
  }
  if (block == 3) {  // LN2 + cross q (into the q slot of qkv)
    g.w = static_cast<const half*>(L.cq_w);
    g.b = static_cast<const half*>(L.cq_b);
    g.n_out = kHidden;
    g.gamma = static_cast<const half*>(L.ln2_g);
    g.beta = static_cast<const half*>(L.ln2_b);
    return launch_bln_gemv<0, 2, false>(g, s);
  }
  if (block == 6) {  // LN3 + fc1 + GELU
    g.w = static_cast<const half*>(L.fc1_w);
    g.b = static_cast<const half*>(L.fc1_b);
    g.out = ffn;
    g.n_out = kFfn;
    g.out_stride = kFfn;
    g.gamma = static_cast<const half*>(L.ln3_g);
    g.beta = static_cast<const half*>(L.ln3_b);
    return launch_bln_gemv<1, 5, false>(g, s);
  }
  BatchFc2Params f{static_cast<const half*>(L.fc2_w), static_cast<const half*>(L.fc2_b), ffn, h, C};
  return launch_bfc2(f, s);
}

}  // namespace fw

extern "C" {

int fw_batch_decoder_step(const fw_batch_decoder_t* d, int steps, fw_stream_t stream) {
  int rc = check_batch_decoder(d);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int step = 0; step < steps; ++step) {
    for (int l = 0; l < d->n_layers; ++l)
      for (int block = 0; block < 8; ++block)
        if ((rc = batch_launch(d, l, block, s))) return rc;
    if ((rc = batch_launch(d, 0, 8, s))) return rc;
  }
  return FW_OK;
}

int fw_batch_decoder_launch(const fw_batch_decoder_t* d, int layer, int block, fw_stream_t stream) {
  int rc = check_batch_decoder(d);
  if (rc) return rc;
  FW_REQUIRE(block >= 0 && block <= 8, FW_ERR_ARG, "batch_decoder_launch: block must be 0..8");
  FW_REQUIRE(block == 8 || (layer >= 0 && layer < d->n_layers), FW_ERR_ARG, "batch_decoder_launch: layer out of range");
  return batch_launch(d, block == 8 ? 0 : layer, block, static_cast<cudaStream_t>(stream));
}

struct fw_decode_loop {
  cudaGraph_t graph;
  cudaGraphExec_t exec;
};

int fw_decode_loop_create(const fw_decoder_t* d, int64_t* ctrl, int steps_per_iter, fw_decode_loop_t** out) {
  int rc = check_decoder(d);
  if (rc) return rc;
  FW_REQUIRE(ctrl != nullptr && out != nullptr, FW_ERR_NULL, "decode_loop_create: ctrl and out are required");
  FW_REQUIRE(steps_per_iter >= 1 && steps_per_iter <= 64, FW_ERR_SHAPE, "decode_loop_create: steps_per_iter must be 1..64");
  *out = nullptr;
  cudaGraph_t graph = nullptr, body = nullptr;
  cudaGraphExec_t exec = nullptr;
  cudaStream_t s = nullptr;
  cudaGraphConditionalHandle handle;
  cudaGraphNode_t init_node = nullptr, loop_node = nullptr;
  cudaError_t e = cudaGraphCreate(&graph, 0);
  if (e == cudaSuccess) e = cudaGraphConditionalHandleCreate(&handle, graph, 0, 0);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
  // node 1: the condition for the first iteration
  if (e == cudaSuccess) e = cudaStreamBeginCaptureToGraph(s, graph, nullptr, nullptr, 0, cudaStreamCaptureModeRelaxed);
  if (e == cudaSuccess) {
    decode_loop_cond_kernel<<<1, 1, 0, s>>>(static_cast<const int64_t*>(d->state), static_cast<const int64_t*>(d->tokens),
                                           ctrl, handle, 1, 1);
    e = cudaGetLastError();
    cudaError_t e2 = cudaStreamEndCapture(s, &graph);
    if (e == cudaSuccess) e = e2;
  }
  if (e == cudaSuccess) {
    size_t n = 1;
    e = cudaGraphGetNodes(graph, &init_node, &n);
  }
  // node 2: WHILE(handle) { steps_per_iter decode steps; condition }
  if (e == cudaSuccess) {
    cudaGraphNodeParams cp = {};
    cp.type = cudaGraphNodeTypeConditional;
    cp.conditional.handle = handle;
    cp.conditional.type = cudaGraphCondTypeWhile;
    cp.conditional.size = 1;
    e = cudaGraphAddNode(&loop_node, graph, &init_node, 1, &cp);
    if (e == cudaSuccess) body = cp.conditional.phGraph_out[0];
  }
  if (e == cudaSuccess) e = cudaStreamBeginCaptureToGraph(s, body, nullptr, nullptr, 0, cudaStreamCaptureModeRelaxed);
  if (e == cudaSuccess) {
    for (int i = 0; i < steps_per_iter && rc == FW_OK; ++i) rc = decoder_one_step(d, s, nullptr);
    if (rc == FW_OK) {
      decode_loop_cond_kernel<<<1, 1, 0, s>>>(static_cast<const int64_t*>(d->state),
                                             static_cast<const int64_t*>(d->tokens), ctrl, handle, 0, steps_per_iter);
      e = cudaGetLastError();
    }
    cudaError_t e2 = cudaStreamEndCapture(s, &body);
    if (e == cudaSuccess) e = e2;
  }
  if (e == cudaSuccess && rc == FW_OK) e = cudaGraphInstantiate(&exec, graph, 0);
  if (s) cudaStreamDestroy(s);
  if (rc != FW_OK || e != cudaSuccess) {
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    if (rc != FW_OK) return rc;
    return set_error(FW_ERR_LAUNCH, "decode_loop_create: %s", cudaGetErrorString(e));
  }
  fw_decode_loop_t* loop = new fw_decode_loop_t{graph, exec};
  *out = loop;
  return FW_OK;
}

int fw_decode_loop_launch(fw_decode_loop_t* loop, fw_stream_t stream) {
  FW_REQUIRE(loop != nullptr, FW_ERR_NULL, "decode_loop_launch: loop is NULL");
  cudaError_t e = cudaGraphLaunch(loop->exec, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? FW_OK : set_error(FW_ERR_LAUNCH, "decode_loop_launch: %s", cudaGetErrorString(e));
}

int fw_decode_loop_destroy(fw_decode_loop_t* loop) {
  if (loop == nullptr) return FW_OK;
  cudaGraphExecDestroy(loop->exec);
  cudaGraphDestroy(loop->graph);
  delete loop;
  return FW_OK;
}

}  // extern "C"
