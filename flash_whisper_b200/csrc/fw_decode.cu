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
#include <mutex>

#include "fw_common.cuh"
#include "fw_host.h"

namespace fw {

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
// because `q` is read as float4 and the persistent kernel keeps an array of four.
struct __align__(16) UnitScratch {
  float q[kHeadDim];
  float sc[kSplitKeys];
  float pacc[4][kHeadDim];
  float red[4];
  float comb_m[kMaxSplits];
  float comb_l[kMaxSplits];
  int last;
};

// Barrier of the 64 threads that process one split: the whole CTA of the stand-alone kernel (id 0)
// or named barrier `id` (a pair of warps) inside the persistent kernel.
__device__ __forceinline__ void unit_sync(int id) {
  if (id == 0)
    __syncthreads();
  else
    asm volatile("bar.sync %0, 64;" ::"r"(id) : "memory");
}

// One 64-key split of one head (whisper_kernels.cu:108-189) on 64 threads, t = 0..63. Thread t
// scores key t over all 64 dims; the 32 pair products fmaf(q0*k0 + q1*k1) are summed in exactly the
// pairing of the reference's warp xor-tree (offsets 16, 8, 4, 2, 1), and the value accumulation keeps
// the reference's per-warp residue classes (keys i = r mod 4, r = 0..3) and their final order, so the
// partial (m, l, acc) is bit-identical to the reference kernel's while the score pass no longer
// serialises a shuffle reduction per key. K rows are read with a per-thread chunk rotation so the
// 16-byte shared loads are bank-conflict free.
__device__ __forceinline__ void attn_unit64(const half* q, const half* ks, const half* vs, int n, float scale, int t,
                                            UnitScratch& U, int sync_id, float* part_acc, float* part_m,
                                            float* part_l) {
  const int lane = t & 31, wa = t >> 5;
  if (t < 32) {
    const float2 qf = __half22float2(__ldcg(reinterpret_cast<const half2*>(q) + t));
    U.q[2 * t] = qf.x;
    U.q[2 * t + 1] = qf.y;
  }
  unit_sync(sync_id);
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
  // value accumulation: warp wa owns residues wa and wa + 2
  float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
  for (int i = wa; i < n; i += 4) {
    const float2 v0 = __half22float2(reinterpret_cast<const half2*>(vs + i * kHeadDim)[lane]);
    const float p0 = U.sc[i];
    acc0.x = fmaf(p0, v0.x, acc0.x);
    acc0.y = fmaf(p0, v0.y, acc0.y);
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
  part_acc[t] = ((U.pacc[0][t] + U.pacc[1][t]) + U.pacc[2][t]) + U.pacc[3][t];
  if (t == 0) {
    *part_m = m;
    *part_l = U.red[2] + U.red[3];
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
    __syncthreads();
    attn_unit64(p.q + head * kHeadDim, ks, vs, n, p.scale, t, U, 0, p.part_acc + static_cast<size_t>(slot) * kHeadDim,
                p.part_m + slot, p.part_l + slot);
  } else if (t == 0) {
    p.part_m[slot] = -INFINITY;
    p.part_l[slot] = 0.f;
  }

  if (p.counters == nullptr) return;
  __threadfence();
  __syncthreads();
  if (t == 0) U.last = atomicAdd(p.counters + head, 1u) == static_cast<unsigned>(splits - 1);
  __syncthreads();
  if (!U.last) return;
  __threadfence();
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
// LM head: fused (optional final LayerNorm) + GEMV over the vocab + argmax (+ optional finalize).
// One CTA per SM owns a contiguous range of vocab rows and streams them through a ring of
// kLmStages shared-memory stages (8 rows each, one row per warp) fed by bulk async copies; the
// first stages are requested before griddepcontrol.wait.
constexpr int kLmStages = 6;
constexpr int kLmRows = 8;
constexpr int kLmStageBytes = kLmRows * kHidden * 2;
constexpr int kLmSmem = kLmStages * kLmStageBytes;

struct LmParams {
  const half* h;
  const half* gamma;
  const half* beta;
  float eps;
  const half* w;
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
  __shared__ __align__(8) uint64_t full[kLmStages];
  __shared__ float red[16];
  __shared__ __align__(16) half ys[kHidden];
  __shared__ unsigned long long warp_best[8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r0 = blockIdx.x * p.rows_per_cta;
  const int r1 = min(p.vocab, r0 + p.rows_per_cta);
  const int nrows = max(0, r1 - r0);
  const int nst = (nrows + kLmRows - 1) / kLmRows;
  const uint64_t policy = policy_evict_first();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kLmStages; ++s) mbar_init(&full[s], 1);
    mbar_fence_init();
    for (int s = 0; s < kLmStages && s < nst; ++s) {
      const int rows = min(kLmRows, nrows - s * kLmRows);
      const unsigned bytes = static_cast<unsigned>(rows) * kHidden * 2;
      mbar_arrive_expect_tx(&full[s], bytes);
      bulk_g2s_stream(smem + s * kLmStageBytes, p.w + static_cast<size_t>(r0 + s * kLmRows) * kHidden, bytes,
                      &full[s], policy);
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
    for (int i = 0; i < 5; ++i) {
      const int idx = threadIdx.x + i * 256;
      ys[idx] = __float2half(ln_apply(v[i], mean, inv, __half2float(p.gamma[idx]), __half2float(p.beta[idx])));
    }
  } else {
#pragma unroll
    for (int i = 0; i < 5; ++i) ys[threadIdx.x + i * 256] = p.h[threadIdx.x + i * 256];
  }
  __syncthreads();
  float xf[40];
  load_x40(ys, xf);

  const bool* mask = p.mask;
  if (kFinalize && p.first_mask && p.prompt_len > 0 && p.state[0] == p.prompt_len - 1) mask = p.first_mask;

  unsigned long long mine = 0;
  for (int s = 0; s < nst; ++s) {
    const int slotb = s % kLmStages;
    if (!mbar_wait(&full[slotb], (s / kLmStages) & 1)) flag_error(FW_DEVERR_TIMEOUT);
    const int row = r0 + s * kLmRows + warp;
    if (row < r1) {
      const uint4* wr = reinterpret_cast<const uint4*>(smem + slotb * kLmStageBytes + warp * kHidden * 2);
      float acc = warp_sum(dot1280_lane(wr, xf));
      acc = round_half(acc);  // logits are fp16 in the reference (whisper_kernels.cu:70-71)
      if (lane == 0 && !(mask && mask[row])) {
        const unsigned long long key = pack_score(acc, row);
        mine = key > mine ? key : mine;
      }
    }
    __syncthreads();
    if (threadIdx.x == 0 && s + kLmStages < nst) {
      const int sn = s + kLmStages;
      const int rows = min(kLmRows, nrows - sn * kLmRows);
      const unsigned bytes = static_cast<unsigned>(rows) * kHidden * 2;
      mbar_arrive_expect_tx(&full[slotb], bytes);
      bulk_g2s_stream(smem + slotb * kLmStageBytes, p.w + static_cast<size_t>(r0 + sn * kLmRows) * kHidden, bytes,
                      &full[slotb], policy);
    }
  }
  if (lane == 0) warp_best[warp] = mine;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long m = 0;
    for (int i = 0; i < 8; ++i) m = warp_best[i] > m ? warp_best[i] : m;
    if (m) atomicMax(p.best, m);
    if (kFinalize) {
      __threadfence();
      const unsigned prev = atomicAdd(p.counter, 1u);
      if (prev == gridDim.x - 1) {
        __threadfence();
        const unsigned long long b = atomicExch(p.best, 0ull);
        finalize_token(b, p.tokens, p.n_tokens, p.state, p.cur, p.max_pos, p.prompt_len);
        *p.counter = 0u;
      }
    }
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
// LayerNorm-prologue GEMV: out[r] = act(W[r] . LN(h) + b[r]) for this CTA's rows. The CTA's
// weight rows (rows_per_cta x 1280 fp16) are bulk-copied into shared memory before the PDL wait.
// kEmbed: h is first built from the token embedding and learned position of the current step
// (custom/model.py:110) and CTA 0 stores it as the residual stream.
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
  // embedding prologue
  const half* embed;
  const half* pos_embed;
  const int64_t* cur;
  const int64_t* state;
  const int64_t* prompt;
  int prompt_len;
  int vocab;
  int max_pos;
  half* h_out;
  // residual GEMV
  const half* x;
  half* h_res;
};

template <bool kEmbed, int kAct>
__global__ void __launch_bounds__(256) ln_gemv_kernel(GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bar;
  __shared__ float red[16];
  __shared__ __align__(16) half ys[kHidden];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r0 = blockIdx.x * p.rows_per_cta;
  const int nr = min(p.rows_per_cta, p.n_out - r0);
  half* ws = reinterpret_cast<half*>(smem);

  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    mbar_fence_init();
    if (nr > 0) {
      mbar_arrive_expect_tx(&bar, static_cast<unsigned>(nr) * kHidden * 2);
      for (int r = 0; r < nr; ++r)
        bulk_g2s(ws + r * kHidden, p.w + static_cast<size_t>(r0 + r) * kHidden, kHidden * 2, &bar);
    }
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();

  float v[5];
  if (kEmbed) {
    int64_t pos = p.state[0];
    int64_t id = (pos >= 0 && pos < p.prompt_len) ? p.prompt[pos] : p.cur[0];
    if (pos < 0 || pos >= p.max_pos || id < 0 || id >= p.vocab) {
      if (threadIdx.x == 0 && blockIdx.x == 0) flag_error(FW_DEVERR_BAD_INDEX);
      pos = pos < 0 ? 0 : (pos >= p.max_pos ? p.max_pos - 1 : pos);
      id = id < 0 ? 0 : (id >= p.vocab ? p.vocab - 1 : id);
    }
    const half* er = p.embed + static_cast<size_t>(id) * kHidden;
    const half* pr = p.pos_embed + static_cast<size_t>(pos) * kHidden;
#pragma unroll
    for (int i = 0; i < 5; ++i) {
      const int idx = threadIdx.x + i * 256;
      v[i] = round_half(__half2float(er[idx]) + __half2float(pr[idx]));
      if (blockIdx.x == 0) p.h_out[idx] = __float2half(v[i]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 5; ++i) v[i] = __half2float(p.h[threadIdx.x + i * 256]);
  }
  float mean, inv;
  ln1280_stats(v, red, p.eps, mean, inv);
#pragma unroll
  for (int i = 0; i < 5; ++i) {
    const int idx = threadIdx.x + i * 256;
    ys[idx] = __float2half(ln_apply(v[i], mean, inv, __half2float(p.gamma[idx]), __half2float(p.beta[idx])));
  }
  __syncthreads();
  float xf[40];
  load_x40(ys, xf);
  if (nr > 0 && !mbar_wait(&bar, 0)) flag_error(FW_DEVERR_TIMEOUT);
  for (int r = warp; r < nr; r += 8) {
    float acc = warp_sum(dot1280_lane(reinterpret_cast<const uint4*>(ws + r * kHidden), xf));
    if (lane == 0) {
      float o = round_half(acc + (p.b ? __half2float(p.b[r0 + r]) : 0.f));
      if (kAct == 1) o = gelu_erf(o);
      p.out[r0 + r] = __float2half(o);
    }
  }
}

// Residual GEMV: h[r] = fp16(h[r] + fp16(W[r] . x + b[r])), x of length k (multiple of 256).
__global__ void __launch_bounds__(256) gemv_residual_kernel(GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bar;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r0 = blockIdx.x * p.rows_per_cta;
  const int nr = min(p.rows_per_cta, p.n_out - r0);
  const int k = p.k;
  half* ws = reinterpret_cast<half*>(smem);
  half* xs = ws + static_cast<size_t>(p.rows_per_cta) * k;

  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    mbar_fence_init();
    if (nr > 0) {
      mbar_arrive_expect_tx(&bar, static_cast<unsigned>(nr) * k * 2);
      for (int r = 0; r < nr; ++r)
        bulk_g2s(ws + static_cast<size_t>(r) * k, p.w + static_cast<size_t>(r0 + r) * k, k * 2, &bar);
    }
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();
  const int kc = k / 8;  // 16-byte chunks
  for (int c = threadIdx.x; c < kc; c += 256)
    reinterpret_cast<uint4*>(xs)[c] = reinterpret_cast<const uint4*>(p.x)[c];
  __syncthreads();
  if (nr > 0 && !mbar_wait(&bar, 0)) flag_error(FW_DEVERR_TIMEOUT);
  for (int r = warp; r < nr; r += 8) {
    const uint4* wr = reinterpret_cast<const uint4*>(ws + static_cast<size_t>(r) * k);
    const uint4* xr = reinterpret_cast<const uint4*>(xs);
    float acc = 0.f;
    for (int c = lane; c < kc; c += 32) {
      const uint4 wv = wr[c], xv = xr[c];
      const half2* pw = reinterpret_cast<const half2*>(&wv);
      const half2* px = reinterpret_cast<const half2*>(&xv);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 fw = __half22float2(pw[j]), fx = __half22float2(px[j]);
        acc = fmaf(fw.x, fx.x, acc);
        acc = fmaf(fw.y, fx.y, acc);
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) {
      const int row = r0 + r;
      const float o = round_half(acc + (p.b ? __half2float(p.b[row]) : 0.f));
      p.h_res[row] = __float2half(__half2float(p.h_res[row]) + o);
    }
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
// Host launchers.
constexpr int kQkvRows = 24;   // 3840 / 24 = 160 CTAs
constexpr int kFc1Rows = 32;   // 5120 / 32 = 160 CTAs
constexpr int kSmallRows = 8;  // 1280 / 8 = 160 CTAs

static int rows_for(int n_out) {
  if (n_out >= 5120) return kFc1Rows;
  if (n_out >= 3840) return kQkvRows;
  return kSmallRows;
}

template <bool kEmbed, int kAct>
static int launch_ln_gemv(const GemvParams& p, cudaStream_t s, bool pdl) {
  const int smem = p.rows_per_cta * kHidden * 2;
  auto kern = ln_gemv_kernel<kEmbed, kAct>;
  cudaError_t e = ensure_smem(kern, smem);
  if (e == cudaSuccess) {
    const int grid = (p.n_out + p.rows_per_cta - 1) / p.rows_per_cta;
    e = launch(kern, dim3(grid), dim3(256), smem, s, pdl, p);
  }
  return launch_status(e, "ln_gemv");
}

static int launch_gemv_residual(const GemvParams& p, cudaStream_t s, bool pdl) {
  const int smem = (p.rows_per_cta + 1) * p.k * 2;
  cudaError_t e = ensure_smem(gemv_residual_kernel, smem);
  if (e == cudaSuccess) {
    const int grid = (p.n_out + p.rows_per_cta - 1) / p.rows_per_cta;
    e = launch(gemv_residual_kernel, dim3(grid), dim3(256), smem, s, pdl, p);
  }
  return launch_status(e, "gemv_residual");
}

static int launch_attention(const AttnParams& p, int heads, int splits, cudaStream_t s, bool pdl) {
  cudaError_t e = launch(attn_split_kernel, dim3(heads, splits), dim3(64), 0, s, pdl, p);
  return launch_status(e, "decode_attention");
}

template <bool kLN, bool kFinalize>
static int launch_lm_head(LmParams p, cudaStream_t s, bool pdl) {
  auto kern = lm_head_kernel<kLN, kFinalize>;
  cudaError_t e = ensure_smem(kern, kLmSmem);
  if (e == cudaSuccess) {
    const int grid = num_sms();
    p.rows_per_cta = (p.vocab + grid - 1) / grid;
    e = launch(kern, dim3(grid), dim3(256), kLmSmem, s, pdl, p);
  }
  return launch_status(e, "lm_head_argmax");
}

// ---------------------------------------------------------------------------------------------
// Split-K attention without caller-allocated workspace (fw_decode_attention_noalloc).
// The fp32 split partials live in this fixed device array instead: per GPU that loads the library,
// kNoAllocMaxSlots head-splits x (64 accumulators + max + sum) x 4 bytes = 528 KB, held until the
// process exits. Host code must not hand the symbol itself to a kernel (on the host it only names
// a stand-in); its device address is looked up once per device with cudaGetSymbolAddress.
constexpr int kNoAllocMaxSlots = 2048;  // heads * ceil(max_len / 64)
static __device__ __align__(256) float g_attn_noalloc_scratch[kNoAllocMaxSlots * (kHeadDim + 2)];

// Device address of g_attn_noalloc_scratch on the current device; looked up on the first call per
// device and cached. Returns nullptr and sets the error message on failure.
static float* noalloc_scratch() {
  static std::mutex mu;
  static float* cached[64] = {nullptr};
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
  if (cached[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error(FW_ERR_LAUNCH, "decode_attention_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      return nullptr;
    }
    cached[dev] = static_cast<float*>(p);
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
  FW_REQUIRE(max_len <= kMaxSplits * kSplitKeys, FW_ERR_SHAPE, "decode_attention: max_len must be <= %d",
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
  return act ? launch_ln_gemv<false, 1>(p, s, false) : launch_ln_gemv<false, 0>(p, s, false);
}

int fw_gemv_residual(const void* x, int k, const void* w, const void* b, void* h, int n_out, fw_stream_t stream) {
  FW_REQUIRE(x && w && h, FW_ERR_NULL, "gemv_residual: x, w and h are required");
  FW_REQUIRE(k > 0 && k % 256 == 0 && k <= 8192, FW_ERR_SHAPE, "gemv_residual: k must be a multiple of 256, <= 8192");
  FW_REQUIRE(n_out > 0, FW_ERR_SHAPE, "gemv_residual: n_out must be positive");
  FW_REQUIRE(aligned16(w) && aligned16(x), FW_ERR_ALIGN, "gemv_residual: w and x must be 16-byte aligned");
  GemvParams p{};
  p.w = static_cast<const half*>(w);
  p.b = static_cast<const half*>(b);
  p.n_out = n_out;
  p.k = k;
  p.rows_per_cta = kSmallRows;
  p.x = static_cast<const half*>(x);
  p.h_res = static_cast<half*>(h);
  return launch_gemv_residual(p, static_cast<cudaStream_t>(stream), false);
}

int fw_decoder_step(const fw_decoder_t* d, int steps, fw_stream_t stream) {
  FW_REQUIRE(d != nullptr, FW_ERR_NULL, "decoder_step: descriptor is NULL");
  FW_REQUIRE(d->n_layers > 0 && d->n_layers <= FW_MAX_LAYERS, FW_ERR_SHAPE, "decoder_step: bad layer count");
  FW_REQUIRE(d->heads * kHeadDim == kHidden, FW_ERR_SHAPE, "decoder_step: heads * 64 must be %d", kHidden);
  FW_REQUIRE(d->max_pos > 0 && d->enc_len > 0 && d->vocab > 0, FW_ERR_SHAPE, "decoder_step: bad sizes");
  FW_REQUIRE(d->embed && d->pos_embed && d->lm_head && d->final_g && d->final_b && d->h && d->qkv && d->attn &&
                 d->cq && d->ffn && d->part_m && d->part_l && d->part_acc && d->counters && d->cur && d->state &&
                 d->tokens && d->best,
             FW_ERR_NULL, "decoder_step: a required pointer is NULL");
  FW_REQUIRE(d->prompt_len == 0 || d->prompt != nullptr, FW_ERR_NULL, "decoder_step: prompt is NULL");
  const int self_splits = (d->max_pos + kSplitKeys - 1) / kSplitKeys;
  const int cross_splits = (d->enc_len + kSplitKeys - 1) / kSplitKeys;
  FW_REQUIRE(self_splits <= kMaxSplits && cross_splits <= kMaxSplits, FW_ERR_SHAPE,
             "decoder_step: max_pos and enc_len must be <= %d", kMaxSplits * kSplitKeys);
  FW_REQUIRE(d->ws_splits >= self_splits && d->ws_splits >= cross_splits, FW_ERR_SHAPE,
             "decoder_step: workspace too small for %d splits", cross_splits);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (steps <= 0) return FW_OK;
  half* h = static_cast<half*>(d->h);
  half* qkv = static_cast<half*>(d->qkv);
  half* attn = static_cast<half*>(d->attn);
  half* cq = static_cast<half*>(d->cq);
  half* ffn = static_cast<half*>(d->ffn);
  for (int step = 0; step < steps; ++step) {
    for (int l = 0; l < d->n_layers; ++l) {
      const fw_decoder_layer_t& L = d->layers[l];
      // LN1 + QKV (+ embedding on layer 0)
      GemvParams g{};
      g.w = static_cast<const half*>(L.qkv_w);
      g.b = static_cast<const half*>(L.qkv_b);
      g.out = qkv;
      g.n_out = 3 * kHidden;
      g.k = kHidden;
      g.rows_per_cta = kQkvRows;
      g.h = h;
      g.gamma = static_cast<const half*>(L.ln1_g);
      g.beta = static_cast<const half*>(L.ln1_b);
      g.eps = d->eps;
      int rc;
      if (l == 0) {
        g.embed = static_cast<const half*>(d->embed);
        g.pos_embed = static_cast<const half*>(d->pos_embed);
        g.cur = d->cur;
        g.state = d->state;
        g.prompt = d->prompt;
        g.prompt_len = d->prompt_len;
        g.vocab = d->vocab;
        g.max_pos = d->max_pos;
        g.h_out = h;
        rc = launch_ln_gemv<true, 0>(g, s, true);
      } else {
        rc = launch_ln_gemv<false, 0>(g, s, true);
      }
      if (rc) return rc;
      // self attention with the fused cache write
      AttnParams a{qkv, static_cast<half*>(L.self_k), static_cast<half*>(L.self_v), qkv + kHidden, qkv + 2 * kHidden,
                   d->state, d->max_pos, d->scale, d->part_m, d->part_l, d->part_acc, attn, d->counters};
      if ((rc = launch_attention(a, d->heads, self_splits, s, true))) return rc;
      // out projection + residual
      GemvParams r{};
      r.w = static_cast<const half*>(L.out_w);
      r.b = static_cast<const half*>(L.out_b);
      r.n_out = kHidden;
      r.k = kHidden;
      r.rows_per_cta = kSmallRows;
      r.x = attn;
      r.h_res = h;
      if ((rc = launch_gemv_residual(r, s, true))) return rc;
      // LN2 + cross q
      g = GemvParams{};
      g.w = static_cast<const half*>(L.cq_w);
      g.b = static_cast<const half*>(L.cq_b);
      g.out = cq;
      g.n_out = kHidden;
      g.k = kHidden;
      g.rows_per_cta = kSmallRows;
      g.h = h;
      g.gamma = static_cast<const half*>(L.ln2_g);
      g.beta = static_cast<const half*>(L.ln2_b);
      g.eps = d->eps;
      if ((rc = launch_ln_gemv<false, 0>(g, s, true))) return rc;
      // cross attention over the encoder states
      AttnParams c{cq, const_cast<half*>(static_cast<const half*>(L.cross_k)),
                   const_cast<half*>(static_cast<const half*>(L.cross_v)), nullptr, nullptr, nullptr, d->enc_len,
                   d->scale, d->part_m, d->part_l, d->part_acc, attn, d->counters};
      if ((rc = launch_attention(c, d->heads, cross_splits, s, true))) return rc;
      r.w = static_cast<const half*>(L.co_w);
      r.b = static_cast<const half*>(L.co_b);
      if ((rc = launch_gemv_residual(r, s, true))) return rc;
      // LN3 + fc1 + GELU
      g = GemvParams{};
      g.w = static_cast<const half*>(L.fc1_w);
      g.b = static_cast<const half*>(L.fc1_b);
      g.out = ffn;
      g.n_out = kFfn;
      g.k = kHidden;
      g.rows_per_cta = kFc1Rows;
      g.h = h;
      g.gamma = static_cast<const half*>(L.ln3_g);
      g.beta = static_cast<const half*>(L.ln3_b);
      g.eps = d->eps;
      if ((rc = launch_ln_gemv<false, 1>(g, s, true))) return rc;
      // fc2 + residual
      r = GemvParams{};
      r.w = static_cast<const half*>(L.fc2_w);
      r.b = static_cast<const half*>(L.fc2_b);
      r.n_out = kHidden;
      r.k = kFfn;
      r.rows_per_cta = kSmallRows;
      r.x = ffn;
      r.h_res = h;
      if ((rc = launch_gemv_residual(r, s, true))) return rc;
    }
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
    int rc = launch_lm_head<true, true>(m, s, true);
    if (rc) return rc;
  }
  return FW_OK;
}

}  // extern "C"
