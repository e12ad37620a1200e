// Whisper encoder on B200: tcgen05/TMEM GEMMs fed by TMA, an implicit-GEMM Conv1d front end,
// row LayerNorm and a tensor-core flash-attention kernel.
//
// The reference runs the HF WhisperEncoder (transformers modeling_whisper.py WhisperEncoder /
// WhisperEncoderLayer: conv1+GELU, conv2+GELU, + sinusoid positions, 32 pre-LN layers, final LN)
// followed by one cross-K/V GEMM for all decoder layers (custom/model.py:143-147). Here:
//
//  * gemm_tc_kernel: C[128 x BN] tile per CTA. Warp 0 issues TMA loads (128B-swizzled K-major
//    tiles) into a STAGES-deep shared-memory ring, warp 1 allocates TMEM and issues
//    tcgen05.mma (M=128, N=BN, K=16, fp16 in / fp32 accumulate in TMEM), warps 2-9 read the
//    accumulator back with tcgen05.ld and run the fused epilogue (bias, GELU, residual add,
//    positions, q scaling, cross-K/V scatter). Weight tiles of the first stages are requested
//    before the PDL wait.
//  * gemm_splitk2_kernel: for long K, a 2-CTA cluster splits K of one 128 x 256 tile and exchanges
//    the fp32 halves over DSMEM before the epilogue.
//  * Conv1d(k=3, pad=1) runs as the same GEMM: the time-major input carries one zero row at each
//    end and a 3-D tensor map [rows/stride, stride, C] lets the producer fetch tap j of output rows
//    t0..t0+127 (input rows stride*t + j) as one box, so no im2col buffer is materialised.
//  * enc_attn_tc_kernel: bidirectional attention, 128 queries x one head per CTA, online softmax
//    over 64-key blocks; S = QK^T and O += PV^T on tcgen05 with S and O in TMEM, Q / K / V^T tiles
//    staged by TMA, two threads per query row for the softmax.
#include <cooperative_groups.h>
#include <cuda.h>

#include "fw_common.cuh"
#include "fw_host.h"

namespace fw {

namespace cg = cooperative_groups;

FW_DEFINE_ERROR_WORD();

__device__ __forceinline__ void enc_flag(unsigned bits) { atomicOr(&g_fw_dev_error, bits); }


// ------------------------------------------------------------------------------------------------
// GEMM
struct GemmEpi {
  const half* bias;
  half* C;
  int64_t ldc;
  const half* R;
  int64_t ldr;
  int M;
  int N;
  int mode;
  float scale;
  int scale_cols;
  int vt_col;  // FW_EPI_QKV_VT: first column written transposed into R
};

__device__ __forceinline__ bool epi_reads_r(int mode) { return mode == FW_EPI_BIAS_RESID || mode == FW_EPI_GELU_POS; }

// One row's 16 columns n..n+15: accumulator bits r, bias from the tile's shared-memory copy sb (8
// halves per uint4, null when the GEMM has none), residual R[row, n..n+15] in ra | rb when the mode
// reads R.
__device__ __forceinline__ void epilogue_store16(const GemmEpi& ep, int row, int n, const uint32_t (&r)[16],
                                                 const uint4* sb, const uint4& ra, const uint4& rb) {
  float o[16];
  float bias[16];
  if (sb != nullptr) {
    const uint4 b0 = sb[0], b1 = sb[1];
    const half* bh0 = reinterpret_cast<const half*>(&b0);
    const half* bh1 = reinterpret_cast<const half*>(&b1);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      bias[j] = __half2float(bh0[j]);
      bias[8 + j] = __half2float(bh1[j]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) bias[j] = 0.f;
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j] = round_half(__uint_as_float(r[j]) + bias[j]);

  if (ep.mode == FW_EPI_QKV_VT && n >= ep.vt_col) {  // V: transposed store, R[(n - vt_col) * ldr + row]
    half* vt = const_cast<half*>(ep.R) + static_cast<size_t>(n - ep.vt_col) * ep.ldr + row;
#pragma unroll
    for (int j = 0; j < 16; ++j) vt[static_cast<size_t>(j) * ep.ldr] = __float2half(o[j]);
    return;
  }
  half* dst;
  if (ep.mode == FW_EPI_CROSS_KV) {
    dst = ep.C + (static_cast<size_t>(n >> 6) * ep.M + row) * 64 + (n & 63);
  } else {
    dst = ep.C + static_cast<size_t>(row) * ep.ldc + n;
  }
  if (ep.mode == FW_EPI_BIAS_GELU) {
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j] = gelu_erf(o[j]);
  } else if (epi_reads_r(ep.mode)) {
    const half* rh0 = reinterpret_cast<const half*>(&ra);
    const half* rh1 = reinterpret_cast<const half*>(&rb);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float res = __half2float(j < 8 ? rh0[j] : rh1[j - 8]);
      o[j] = ep.mode == FW_EPI_GELU_POS ? round_half(gelu_erf(o[j])) + res : res + o[j];
    }
  } else if (ep.mode == FW_EPI_BIAS_SCALE || ep.mode == FW_EPI_QKV_VT) {
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (n + j < ep.scale_cols) o[j] = o[j] * ep.scale;
  }
  uint4 w0, w1;
  half2* h0 = reinterpret_cast<half2*>(&w0);
  half2* h1 = reinterpret_cast<half2*>(&w1);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    h0[j] = __floats2half2_rn(o[2 * j], o[2 * j + 1]);
    h1[j] = __floats2half2_rn(o[8 + 2 * j], o[8 + 2 * j + 1]);
  }
  reinterpret_cast<uint4*>(dst)[0] = w0;
  reinterpret_cast<uint4*>(dst)[1] = w1;
}

// Persistent warp-specialised GEMM. CTA b processes output tiles b, b + gridDim.x, ... in n-major
// order (tile t covers m tile t % m_tiles and n tile t / m_tiles), so the CTAs that run together
// share weight (B) slices. Warp 0 streams A and B k-blocks through a STAGES-deep ring (the B
// tiles of the first stages are requested before the PDL wait), warp 1 issues the MMAs into one of
// kAccBufs TMEM accumulators, warps 2-9 drain the previous accumulator through the epilogue while
// the next tile's MMAs run. BN = kSub * kSubN columns per tile: kSub MMAs of N = kSubN per K step.
constexpr int kGemmEpiWarps = 8;  // two per TMEM lane quadrant, each draining half of the columns
constexpr int kGemmThreads = 32 * (2 + kGemmEpiWarps);

template <int kSubN, int kSub, int STAGES, bool kConv>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                                                         const __grid_constant__ CUtensorMap tmB, int num_kb,
                                                         int conv_c, int conv_stride, GemmEpi ep, int m_tiles,
                                                         int n_tiles, const char* l2_next, unsigned l2_bytes) {
  constexpr int BM = 128, BK = 64;
  constexpr int BN = kSubN * kSub;
  constexpr uint32_t kABytes = BM * BK * 2;
  constexpr uint32_t kBSubBytes = kSubN * BK * 2;
  constexpr uint32_t kBBytes = BN * BK * 2;
  constexpr uint32_t kStageBytes = kABytes + kBBytes;
  constexpr int kAccBufs = 2 * BN <= 512 ? 2 : 1;
  constexpr uint32_t kTmemCols = BN * kAccBufs <= 64 ? 64 : BN * kAccBufs <= 128 ? 128 : BN * kAccBufs <= 256 ? 256 : 512;
  static_assert(BN * kAccBufs <= 512, "accumulators exceed TMEM");
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t acc_full[kAccBufs];
  __shared__ __align__(8) uint64_t acc_empty[kAccBufs];
  __shared__ uint32_t tmem_base_sh;
  __shared__ __align__(16) uint4 s_bias[2][BN / 8];

  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = m_tiles * n_tiles;
  const int first = blockIdx.x;
  const int pre = num_kb < STAGES ? num_kb : STAGES;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < kAccBufs; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kGemmEpiWarps);
    }
    mbar_fence_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (first < tiles) {  // weight tiles of the first stages do not depend on the previous kernel
      const int n0 = (first / m_tiles) * BN;
      for (int kb = 0; kb < pre; ++kb) {
        mbar_arrive_expect_tx(&full_bar[kb], kStageBytes);
#pragma unroll
        for (int j = 0; j < kSub; ++j)
          tma_load_2d(smem + kb * kStageBytes + kABytes + j * kBSubBytes, &tmB, &full_bar[kb], kb * BK,
                      n0 + j * kSubN);
      }
    }
    // warm L2 with this CTA's share of the weights of the next GEMM
    if (l2_next != nullptr && l2_bytes > 0) {
      const unsigned share = ((l2_bytes + gridDim.x - 1) / gridDim.x + 15u) & ~15u;
      const unsigned off = share * blockIdx.x;
      if (off < l2_bytes) {
        const unsigned n = min(share, l2_bytes - off);
        for (unsigned o = 0; o < n; o += 65536u) l2_prefetch(l2_next + off + o, min(65536u, n - o));
      }
    }
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_sh, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;

  if (warp == 0) {
    if (lane == 0) {
      pdl_wait();
      pdl_trigger();
      int it = 0;  // k-block counter across tiles (ring position)
      for (int t = first; t < tiles; t += gridDim.x) {
        const int m0 = (t % m_tiles) * BM, n0 = (t / m_tiles) * BN;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          uint8_t* sa = smem + s * kStageBytes;
          const bool b_loaded = t == first && kb < pre;
          if (!b_loaded) {
            if (it >= STAGES && !mbar_wait(&empty_bar[s], ph ^ 1u)) {
              enc_flag(FW_DEVERR_TIMEOUT);
              t = tiles;
              break;
            }
            mbar_arrive_expect_tx(&full_bar[s], kStageBytes);
#pragma unroll
            for (int j = 0; j < kSub; ++j)
              tma_load_2d(sa + kABytes + j * kBSubBytes, &tmB, &full_bar[s], kb * BK, n0 + j * kSubN);
          }
          if (kConv) {
            const int k = kb * BK;
            const int tap = k / conv_c;
            const int c0 = k - tap * conv_c;
            tma_load_3d(sa, &tmA, &full_bar[s], c0, tap % conv_stride, m0 + tap / conv_stride);
          } else {
            tma_load_2d(sa, &tmA, &full_bar[s], kb * BK, m0);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16(BM, kSubN);
      int it = 0, local = 0;
      for (int t = first; t < tiles; t += gridDim.x, ++local) {
        const int buf = local % kAccBufs;
        const uint32_t use = local / kAccBufs;
        if (local >= kAccBufs && !mbar_wait(&acc_empty[buf], (use - 1) & 1u)) {  // epilogue drained it
          enc_flag(FW_DEVERR_TIMEOUT);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(buf * BN);
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!mbar_wait(&full_bar[s], ph)) {
            enc_flag(FW_DEVERR_TIMEOUT);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = base + s * kStageBytes;
          const uint64_t adesc = sw128_desc(a_addr);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
#pragma unroll
            for (int j = 0; j < kSub; ++j)
              tc_mma_f16(d + j * kSubN, adesc + 2 * kk, sw128_desc(a_addr + kABytes + j * kBSubBytes) + 2 * kk, idesc,
                         (kb | kk) != 0 ? 1u : 0u);
          }
          tc_commit(&empty_bar[s]);
        }
        tc_commit(&acc_full[buf]);
        if (!ok) break;
      }
    }
  } else {
    // Epilogue warps 2..9: warp w reads TMEM lanes 32 (w % 4) .. + 31 (its rows) and the 32-column
    // chunks c with (c / 32) % 2 == (w - 2) / 4. What does not depend on the accumulator is fetched
    // while the tile's MMAs run: the tile's bias slice into shared memory (double-buffered by tile,
    // one named barrier of the epilogue threads per tile) and this row's residual for the first
    // chunk; the residual of the next chunk is loaded while the current one is processed.
    pdl_wait();
    const int q = warp & 3;
    const int half_id = (warp - 2) >> 2;
    const int et = threadIdx.x - 64;
    const bool reads_r = epi_reads_r(ep.mode);
    bool failed = false;
    int local = 0;
    for (int t = first; t < tiles; t += gridDim.x, ++local) {
      const int buf = local % kAccBufs;
      const uint32_t use = local / kAccBufs;
      const int m0 = (t % m_tiles) * BM, n0 = (t / m_tiles) * BN;
      const int row = m0 + q * 32 + lane;
      const bool row_ok = row < ep.M;
      uint4* sb = s_bias[local & 1];
      if (ep.bias != nullptr) {
        const uint4* b4 = reinterpret_cast<const uint4*>(ep.bias + n0);
        for (int i = et; i < BN / 8; i += 32 * kGemmEpiWarps) sb[i] = __ldg(b4 + i);
      }
      const uint4* r4 = reinterpret_cast<const uint4*>(ep.R + (row_ok ? static_cast<size_t>(row) * ep.ldr : 0) + n0);
      const bool load_r = reads_r && row_ok;
      uint4 cur[4] = {}, nxt[4] = {};
      if (load_r) {
#pragma unroll
        for (int i = 0; i < 4; ++i) cur[i] = r4[half_id * 4 + i];
      }
      // Every epilogue warp reaches this barrier once per tile, also after a timed-out wait (it then
      // skips the tile), so no warp can be left waiting here.
      asm volatile("bar.sync 1, %0;" ::"r"(32 * kGemmEpiWarps) : "memory");  // bias slice visible
      const uint4* sbias = ep.bias != nullptr ? sb : nullptr;
      if (failed || !mbar_wait_warp(&acc_full[buf], use & 1u)) {
        if (!failed) enc_flag(FW_DEVERR_TIMEOUT);
        failed = true;
        continue;
      }
      tc_fence_after();
      const uint32_t d = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * BN);
#pragma unroll 1
      for (int c = half_id * 32; c < BN; c += 64) {
        uint32_t r0[16], r1[16];
        tc_ld16(d + static_cast<uint32_t>(c), r0);
        tc_ld16(d + static_cast<uint32_t>(c + 16), r1);
        if (load_r && c + 64 < BN) {
#pragma unroll
          for (int i = 0; i < 4; ++i) nxt[i] = r4[(c + 64) / 8 + i];
        }
        tc_wait_ld();
        if (row_ok) {
          epilogue_store16(ep, row, n0 + c, r0, sbias ? sbias + c / 8 : nullptr, cur[0], cur[1]);
          epilogue_store16(ep, row, n0 + c + 16, r1, sbias ? sbias + c / 8 + 2 : nullptr, cur[2], cur[3]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) cur[i] = nxt[i];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------------------------------------
// Split-K GEMM for long K: a cluster of two CTAs computes one 128 x 256 tile, CTA r accumulating
// k-blocks r * num_kb / 2 .. (r + 1) * num_kb / 2 - 1 in its own TMEM (N = 256 MMAs). After both
// mainloops each CTA writes the 128 columns its peer finishes (fp32, column-major 128 x 128, 64 KB)
// into the peer's now idle stage ring through DSMEM; after a second cluster barrier each CTA adds
// the received half to its own and runs the epilogue on its 128 columns. One tile per cluster, one
// round (the dispatcher uses it only when 2 x tiles CTAs fit on the GPU).
template <int STAGES, bool kConv>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_splitk2_kernel(const __grid_constant__ CUtensorMap tmA,
                                                              const __grid_constant__ CUtensorMap tmB, int num_kb,
                                                              int conv_c, int conv_stride, GemmEpi ep, int m_tiles,
                                                              const char* l2_next, unsigned l2_bytes) {
  constexpr int BM = 128, BK = 64, BN = 256, kHalf = BN / 2;
  constexpr uint32_t kABytes = BM * BK * 2;
  constexpr uint32_t kBBytes = BN * BK * 2;
  constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static_assert(STAGES * kStageBytes >= kHalf * BM * 4, "the exchange buffer lives in the stage ring");
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t acc_full;
  __shared__ uint32_t tmem_base_sh;
  __shared__ __align__(16) uint4 s_bias[kHalf / 8];

  cg::cluster_group cluster = cg::this_cluster();
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw);
  float* xbuf = reinterpret_cast<float*>(smem);  // after the mainloop: [kHalf columns][BM rows] from the peer
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = static_cast<int>(cluster.block_rank());
  const int peer = rank ^ 1;
  const int tile = static_cast<int>(blockIdx.x) >> 1;
  const int m0 = (tile % m_tiles) * BM, n0 = (tile / m_tiles) * BN;
  const int nkb = num_kb / 2, kb0 = rank * nkb;
  const int pre = nkb < STAGES ? nkb : STAGES;

  if (warp == 0 && lane == 0) {
    for (int st = 0; st < STAGES; ++st) {
      mbar_init(&full_bar[st], 1);
      mbar_init(&empty_bar[st], 1);
    }
    mbar_init(&acc_full, 1);
    mbar_fence_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    for (int i = 0; i < pre; ++i) {  // weight tiles of the first stages do not depend on the previous kernel
      mbar_arrive_expect_tx(&full_bar[i], kStageBytes);
      tma_load_2d(smem + i * kStageBytes + kABytes, &tmB, &full_bar[i], (kb0 + i) * BK, n0);
    }
    if (l2_next != nullptr && l2_bytes > 0) {
      const unsigned share = ((l2_bytes + gridDim.x - 1) / gridDim.x + 15u) & ~15u;
      const unsigned off = share * blockIdx.x;
      if (off < l2_bytes) {
        const unsigned n = min(share, l2_bytes - off);
        for (unsigned o = 0; o < n; o += 65536u) l2_prefetch(l2_next + off + o, min(65536u, n - o));
      }
    }
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_sh, BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;

  // epilogue-thread state prepared while the mainloop runs
  const int q = warp & 3, hid = (warp - 2) >> 2;  // warps 2..9: TMEM lane quadrant, 64-column half
  const int row = m0 + q * 32 + lane;
  const bool row_ok = warp >= 2 && row < ep.M;
  uint4 res[8] = {};
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {
      pdl_wait();
      pdl_trigger();
      for (int i = 0; i < nkb; ++i) {
        const int st = i % STAGES;
        const uint32_t ph = (i / STAGES) & 1u;
        uint8_t* sa = smem + st * kStageBytes;
        if (i >= pre) {
          if (!mbar_wait(&empty_bar[st], ph ^ 1u)) {
            enc_flag(FW_DEVERR_TIMEOUT);
            break;
          }
          mbar_arrive_expect_tx(&full_bar[st], kStageBytes);
          tma_load_2d(sa + kABytes, &tmB, &full_bar[st], (kb0 + i) * BK, n0);
        }
        if (kConv) {
          const int k = (kb0 + i) * BK;
          const int tap = k / conv_c;
          const int c0 = k - tap * conv_c;
          tma_load_3d(sa, &tmA, &full_bar[st], c0, tap % conv_stride, m0 + tap / conv_stride);
        } else {
          tma_load_2d(sa, &tmA, &full_bar[st], (kb0 + i) * BK, m0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16(BM, BN);
      for (int i = 0; i < nkb; ++i) {
        const int st = i % STAGES;
        if (!mbar_wait(&full_bar[st], (i / STAGES) & 1u)) {
          enc_flag(FW_DEVERR_TIMEOUT);
          break;
        }
        tc_fence_after();
        const uint32_t a_addr = base + st * kStageBytes;
        const uint64_t adesc = sw128_desc(a_addr), bdesc = sw128_desc(a_addr + kABytes);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) tc_mma_f16(tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (i | kk) != 0);
        tc_commit(&empty_bar[st]);
      }
      tc_commit(&acc_full);
    }
  } else {
    pdl_wait();
    const int et = threadIdx.x - 64;
    if (ep.bias != nullptr && et < kHalf / 8)
      s_bias[et] = __ldg(reinterpret_cast<const uint4*>(ep.bias + n0 + rank * kHalf) + et);
    if (row_ok && epi_reads_r(ep.mode)) {
      const uint4* r4 = reinterpret_cast<const uint4*>(ep.R + static_cast<size_t>(row) * ep.ldr + n0 + rank * kHalf +
                                                       hid * 64);
#pragma unroll
      for (int i = 0; i < 8; ++i) res[i] = r4[i];
    }
    ok = mbar_wait_warp(&acc_full, 0);
    if (!ok) enc_flag(FW_DEVERR_TIMEOUT);
  }
  // 1: both CTAs' MMAs are complete (every epilogue warp saw acc_full), so both stage rings are idle
  tc_fence_before();
  cluster.sync();
  tc_fence_after();
  if (warp >= 2 && ok) {
    float* px = cluster.map_shared_rank(xbuf, peer);
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
#pragma unroll 1
    for (int p4 = 0; p4 < 4; ++p4) {
      const int c = hid * 64 + p4 * 16;  // column within the peer's half
      uint32_t r[16];
      tc_ld16(lane_base + static_cast<uint32_t>(peer * kHalf + c), r);
      tc_wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) px[(c + j) * BM + q * 32 + lane] = __uint_as_float(r[j]);
    }
  }
  // 2: the peer's partial of this CTA's columns is in xbuf
  tc_fence_before();
  cluster.sync();
  tc_fence_after();
  if (warp >= 2 && ok) {
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
#pragma unroll
    for (int p4 = 0; p4 < 4; ++p4) {
      const int c = hid * 64 + p4 * 16;  // column within this CTA's half
      uint32_t r[16];
      tc_ld16(lane_base + static_cast<uint32_t>(rank * kHalf + c), r);
      tc_wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j)
        r[j] = __float_as_uint(__uint_as_float(r[j]) + xbuf[(c + j) * BM + q * 32 + lane]);
      if (row_ok)
        epilogue_store16(ep, row, n0 + rank * kHalf + c, r, ep.bias != nullptr ? s_bias + c / 8 : nullptr,
                         res[2 * p4], res[2 * p4 + 1]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, BN);
  }
}

// ------------------------------------------------------------------------------------------------
// Row LayerNorm: one warp per row, cols % 256 == 0 (<= 2048), two-pass variance in fp32.
__global__ void __launch_bounds__(256) layernorm_rows_kernel(const half* __restrict__ x, const half* __restrict__ g,
                                                             const half* __restrict__ b, half* __restrict__ y,
                                                             int rows, int cols, float eps) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nc = cols / 256;  // 16-byte chunks per lane
  // gamma and beta are weights: loaded before the wait
  uint4 gw[8], bw[8];
  const uint4* g4 = reinterpret_cast<const uint4*>(g);
  const uint4* b4 = reinterpret_cast<const uint4*>(b);
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    if (c < nc) {
      gw[c] = __ldg(g4 + lane + 32 * c);
      bw[c] = __ldg(b4 + lane + 32 * c);
    }
  }
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x * 8 + warp;
  if (row >= rows) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<size_t>(row) * cols);
  float v[64];
  float sum = 0.f;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    if (c < nc) {
      const uint4 u = xr[lane + 32 * c];
      const half* hv = reinterpret_cast<const half*>(&u);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[c * 8 + j] = __half2float(hv[j]);
        sum += v[c * 8 + j];
      }
    }
  }
  sum = warp_sum(sum);
  const float mean = sum / cols;
  float sq = 0.f;
#pragma unroll
  for (int c = 0; c < 8; ++c)
    if (c < nc)
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = v[c * 8 + j] - mean;
        sq = fmaf(d, d, sq);
      }
  sq = warp_sum(sq);
  const float inv = rsqrtf(sq / cols + eps);
  uint4* yr = reinterpret_cast<uint4*>(y + static_cast<size_t>(row) * cols);
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    if (c < nc) {
      const half* gh = reinterpret_cast<const half*>(&gw[c]);
      const half* bh = reinterpret_cast<const half*>(&bw[c]);
      uint4 out;
      half* oh = reinterpret_cast<half*>(&out);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        oh[j] = __float2half(fmaf((v[c * 8 + j] - mean) * inv, __half2float(gh[j]), __half2float(bh[j])));
      yr[lane + 32 * c] = out;
    }
  }
}

// ------------------------------------------------------------------------------------------------
// Encoder attention on tcgen05 (bidirectional, one head, kAttnQ queries per CTA, 64-key blocks).
//   warp 0 (one lane): TMA loads - Q once, then K and V^T blocks through a kAttnStages ring
//   warp 1 (one lane): S = Q K^T into TMEM, then O += P V into TMEM, one 64-key block at a time;
//                      S of block j + 1 is issued as soon as the softmax has read S of block j
//   warps 2-9: two threads per query row (TMEM lane), warp w taking keys 32 ((w - 2) / 4) .. + 31
//              of each block for the rows of TMEM lane quadrant w % 4: online softmax of S (exp2,
//              running max and sum in fp32), P as fp16 into one of two 128B-swizzled K-major shared
//              tiles (the A operand of the P V MMA), and the final O / l store (each warp 32 of the
//              64 output columns). Both threads of a row take the max over all 64 scores of the
//              block (the same value, so the same rescale decisions without an exchange); each
//              sums its own keys and the two sums are added once at the end. The max used for P
//              moves only when a row's block max exceeds it by more than 2^8 (P <= 256 in fp16),
//              and only then is the O row in TMEM rescaled; so the softmax of block j waits for
//              P V of block j - 2 (its P buffer), not j - 1, and P V overlaps the next block's
//              softmax.
// V is read transposed ([heads * 64, seq_pad], keys contiguous) so both MMAs use K-major operands.
// q arrives pre-scaled by 1/8 (HF WhisperAttention), so S is used unscaled.
__device__ __forceinline__ void tc_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

constexpr int kAttnQ = 128;
constexpr int kAttnK = 64;
constexpr int kAttnStages = 3;
constexpr uint32_t kAttnQBytes = kAttnQ * 64 * 2;   // 16 KB
constexpr uint32_t kAttnKBytes = kAttnK * 64 * 2;   // 8 KB
constexpr uint32_t kAttnPBytes = kAttnQ * kAttnK * 2;  // 16 KB
constexpr int kAttnSmem = kAttnQBytes + 2 * kAttnStages * kAttnKBytes + 2 * kAttnPBytes + 1024;
constexpr int kAttnSoftWarps = 8;  // two per TMEM lane quadrant, each half of a block's keys
constexpr int kAttnThreads = 32 * (2 + kAttnSoftWarps);

__global__ void __launch_bounds__(kAttnThreads, 2) enc_attn_tc_kernel(const __grid_constant__ CUtensorMap tmQK,
                                                                      const __grid_constant__ CUtensorMap tmVt,
                                                                      int kcol, half* __restrict__ out, int ldo,
                                                                      int seq) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bar_q, full_k[kAttnStages], empty_k[kAttnStages], full_v[kAttnStages],
      empty_v[kAttnStages], s_full[2], s_free[2], p_full[2], o_done[2], l_bar;
  __shared__ float s_l[2][kAttnQ];  // each row's two partial sums (key halves 0 and 1)
  __shared__ uint32_t tmem_base_sh;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw);
  uint8_t* qs = smem;
  uint8_t* ks = smem + kAttnQBytes;
  uint8_t* vts = ks + kAttnStages * kAttnKBytes;
  uint8_t* ps = vts + kAttnStages * kAttnKBytes;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = blockIdx.y;
  const int q0 = blockIdx.x * kAttnQ;
  const int nkb = (seq + kAttnK - 1) / kAttnK;

  if (warp == 0 && lane == 0) {
    mbar_init(&bar_q, 1);
    for (int i = 0; i < kAttnStages; ++i) {
      mbar_init(&full_k[i], 1);
      mbar_init(&empty_k[i], 1);
      mbar_init(&full_v[i], 1);
      mbar_init(&empty_v[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);                // S buffer i holds the block's scores (block j uses buffer j & 1)
      mbar_init(&s_free[i], kAttnSoftWarps);   // the softmax has read S buffer i
      mbar_init(&p_full[i], kAttnSoftWarps);   // P buffer i full (block j uses buffer j & 1)
      mbar_init(&o_done[i], 1);                // P V of the last block that used buffer i complete
    }
    mbar_init(&l_bar, 32 * kAttnSoftWarps);  // every softmax thread has stored its partial sum
    mbar_fence_init();
    tma_prefetch_desc(&tmQK);
    tma_prefetch_desc(&tmVt);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_sh, 256);  // S: columns 0-63 and 64-127 (two blocks), O: columns 128-191
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(&bar_q, kAttnQBytes);
      tma_load_2d(qs, &tmQK, &bar_q, head * 64, q0);  // the map's box is 64 rows: Q is two boxes
      tma_load_2d(qs + kAttnKBytes, &tmQK, &bar_q, head * 64, q0 + 64);
      for (int j = 0; j < nkb; ++j) {
        const int st = j % kAttnStages;
        const uint32_t ph = (j / kAttnStages) & 1u;
        if (j >= kAttnStages && !mbar_wait(&empty_k[st], ph ^ 1u)) {
          enc_flag(FW_DEVERR_TIMEOUT);
          break;
        }
        mbar_arrive_expect_tx(&full_k[st], kAttnKBytes);
        tma_load_2d(ks + st * kAttnKBytes, &tmQK, &full_k[st], kcol + head * 64, j * kAttnK);
        if (j >= kAttnStages && !mbar_wait(&empty_v[st], ph ^ 1u)) {
          enc_flag(FW_DEVERR_TIMEOUT);
          break;
        }
        mbar_arrive_expect_tx(&full_v[st], kAttnKBytes);
        tma_load_2d(vts + st * kAttnKBytes, &tmVt, &full_v[st], j * kAttnK, head * 64);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16(kAttnQ, 64);  // S: N = 64 keys; O: N = 64 dims
      const uint32_t o_tmem = tmem + 128;
      bool ok = mbar_wait(&bar_q, 0);
      auto issue_s = [&](int j) {  // S_j = Q K_j^T into S buffer j & 1
        const int st = j % kAttnStages;
        if (!mbar_wait(&full_k[st], (j / kAttnStages) & 1u)) return false;
        tc_fence_after();
        const uint64_t ad = sw128_desc(base), bd = sw128_desc(smem_u32(ks + st * kAttnKBytes));
        const uint32_t s_tmem = tmem + static_cast<uint32_t>((j & 1) * 64);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) tc_mma_f16(s_tmem, ad + 2 * kk, bd + 2 * kk, idesc, kk != 0 ? 1u : 0u);
        tc_commit(&empty_k[st]);
        tc_commit(&s_full[j & 1]);
        return true;
      };
      if (ok) ok = issue_s(0);
      if (ok && nkb > 1) ok = issue_s(1);
      for (int j = 0; ok && j < nkb; ++j) {
        // S_{j+2} reuses S buffer j & 1 once the softmax has read S_j
        if (j + 2 < nkb) {
          if (!mbar_wait(&s_free[j & 1], (j >> 1) & 1u)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (!(ok = issue_s(j + 2))) break;
        }
        // O += P_j V_j
        const int st = j % kAttnStages;
        if (!mbar_wait(&p_full[j & 1], (j >> 1) & 1u) || !mbar_wait(&full_v[st], (j / kAttnStages) & 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t ad = sw128_desc(smem_u32(ps + (j & 1) * kAttnPBytes));
        const uint64_t bd = sw128_desc(smem_u32(vts + st * kAttnKBytes));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc_mma_f16(o_tmem, ad + 2 * kk, bd + 2 * kk, idesc, (j | kk) != 0 ? 1u : 0u);
        tc_commit(&empty_v[st]);
        tc_commit(&o_done[j & 1]);
      }
      if (!ok) enc_flag(FW_DEVERR_TIMEOUT);
    }
  } else {
    const int q = warp & 3;            // TMEM lanes 32q..32q+31
    const int hs = (warp - 2) >> 2;    // this warp's keys 32 hs .. 32 hs + 31 of each block
    const int r = q * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
    constexpr float kLog2e = 1.4426950408889634f;
    constexpr float kGrow = 8.f;  // log2 units: the max used for P lags the true max by at most this
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkb; ++j) {
      if (!mbar_wait_warp(&s_full[j & 1], (j >> 1) & 1u)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sv[32], so[32];  // this warp's keys, the other half's keys (only for the row max)
      {
        const uint32_t sb = lane_base + (j & 1) * 64;
        uint32_t u[4][16];
        tc_ld16(sb + hs * 32, u[0]);
        tc_ld16(sb + hs * 32 + 16, u[1]);
        tc_ld16(sb + (hs ^ 1) * 32, u[2]);
        tc_ld16(sb + (hs ^ 1) * 32 + 16, u[3]);
        tc_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          sv[i] = __uint_as_float(u[0][i]);
          sv[16 + i] = __uint_as_float(u[1][i]);
          so[i] = __uint_as_float(u[2][i]);
          so[16 + i] = __uint_as_float(u[3][i]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[j & 1]);  // S buffer j & 1 may now take block j + 2
      const int kvalid = seq - j * kAttnK;
      if (kvalid < kAttnK) {  // the ragged last block (the same for every thread of the CTA)
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if (hs * 32 + i >= kvalid) sv[i] = -INFINITY;
          if ((hs ^ 1) * 32 + i >= kvalid) so[i] = -INFINITY;
        }
      }
      // Row max over all 64 keys, four independent chains; fmax is exact, so both warps of a row
      // get the same value whichever half they hold.
      float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        mq[i & 3] = fmaxf(mq[i & 3], sv[i]);
        mq[(i + 2) & 3] = fmaxf(mq[(i + 2) & 3], so[i]);
      }
      const float mb = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3])) * kLog2e;
      // The TMEM accesses of a rescale need the whole warp: it happens when any row's max grew by
      // more than kGrow (always on the first block, where m = -inf); rows whose max did not grow get
      // corr = 1 exactly.
      const bool rescale = __any_sync(0xffffffffu, mb > m + kGrow);
      float corr = 1.f;
      if (rescale) {
        const float m_new = fmaxf(m, mb);
        corr = fast_exp2(m - m_new);  // 0 on the first block
        m = m_new;
      }
      float sq[4] = {0.f, 0.f, 0.f, 0.f};  // four independent sum chains
      uint32_t pk[16];
      const float nm = -m;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float p0 = fast_exp2(fmaf(sv[2 * i], kLog2e, nm)), p1 = fast_exp2(fmaf(sv[2 * i + 1], kLog2e, nm));
        sq[i & 3] += p0 + p1;
        half2 h2 = __floats2half2_rn(p0, p1);
        pk[i] = *reinterpret_cast<uint32_t*>(&h2);
      }
      l = l * corr + ((sq[0] + sq[1]) + (sq[2] + sq[3]));
      // P buffer j & 1 is free once P V of block j - 2 has completed
      if (j >= 2 && !mbar_wait_warp(&o_done[j & 1], ((j >> 1) - 1) & 1u)) {
        ok = false;
        break;
      }
      if (rescale && j > 0) {  // O holds P V of blocks 0 .. j - 1 once block j - 1's has completed
        if (!mbar_wait_warp(&o_done[(j - 1) & 1], ((j - 1) >> 1) & 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t u[2][16];  // this warp's 32 of the 64 O columns
#pragma unroll
        for (int c = 0; c < 2; ++c) tc_ld16(lane_base + 128 + hs * 32 + c * 16, u[c]);
        tc_wait_ld();
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int i = 0; i < 16; ++i) u[c][i] = __float_as_uint(__uint_as_float(u[c][i]) * corr);
#pragma unroll
        for (int c = 0; c < 2; ++c) tc_st16(lane_base + 128 + hs * 32 + c * 16, u[c]);
        tc_wait_st();
      }
      // P row r: 8 chunks of 16 bytes, chunk c at r * 128 + ((c ^ (r & 7)) * 16) (128B swizzle);
      // this warp writes chunks 4 hs .. 4 hs + 3 (its 32 keys)
      uint8_t* pb = ps + (j & 1) * kAttnPBytes;
#pragma unroll
      for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(pb + r * 128 + (((hs * 4 + c) ^ (r & 7)) << 4)) =
            make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      fence_proxy_async_shared();  // generic-proxy P stores -> tensor-core reads
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[j & 1]);
    }
    // Row sum = the two halves' partial sums (every softmax thread stores and arrives exactly once,
    // also after a timed-out wait, so the bounded wait below only fails if a warp never got here).
    s_l[hs][r] = l;
    mbar_arrive(&l_bar);
    // the last block's P V completes after every earlier MMA of this CTA
    if (ok && nkb > 0 && mbar_wait_warp(&o_done[(nkb - 1) & 1], ((nkb - 1) >> 1) & 1u) &&
        mbar_wait_warp(&l_bar, 0)) {
      tc_fence_after();
      const float inv = 1.f / (s_l[0][r] + s_l[1][r]);
      const int row = q0 + r;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t u[16];
        tc_ld16(lane_base + 128 + hs * 32 + c * 16, u);
        tc_wait_ld();
        if (row < seq) {
          uint4 w[2];
          half2* h = reinterpret_cast<half2*>(w);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            h[i] = __floats2half2_rn(__uint_as_float(u[2 * i]) * inv, __uint_as_float(u[2 * i + 1]) * inv);
          uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(row) * ldo + head * 64 + hs * 32 + c * 16);
          dst[0] = w[0];
          dst[1] = w[1];
        }
      }
    } else {
      enc_flag(FW_DEVERR_TIMEOUT);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// V^T [heads * 64, ldv] (keys contiguous) from the v columns of a [seq, ld] q|k|v buffer, for the
// stand-alone attention entry point (the encoder writes V^T straight from the QKV GEMM epilogue).
__global__ void __launch_bounds__(256) transpose_v_kernel(const half* __restrict__ qkv, int64_t ld, int vcol,
                                                          half* __restrict__ vt, int64_t ldv, int seq, int cols) {
  __shared__ half tile[32][33];
  const int t0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  pdl_wait();
  pdl_trigger();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int t = t0 + i, c = c0 + threadIdx.x;
    tile[i][threadIdx.x] = (t < seq && c < cols) ? qkv[static_cast<size_t>(t) * ld + vcol + c] : __float2half(0.f);
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int c = c0 + i, t = t0 + threadIdx.x;
    if (c < cols && t < seq) vt[static_cast<size_t>(c) * ldv + t] = tile[threadIdx.x][i];
  }
}

// ------------------------------------------------------------------------------------------------
// Host side
// 2-D fp16 map [outer][inner] with row stride `ld` elements, box {64, box_outer}, 128B swizzle.
static int make_map_2d(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld,
                       uint32_t box_outer) {
  EncodeTiledFn enc = tensor_map_encode_fn();
  if (!enc) return set_error(FW_ERR_LAUNCH, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {64, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(FW_ERR_ARG, "tensor map encode failed (%d)", static_cast<int>(r));
  return FW_OK;
}

// 3-D fp16 map over a padded time-major conv input [rows][C] viewed as [rows/stride][stride][C],
// box {64, 1, 128}.
static int make_map_conv(CUtensorMap* m, const void* ptr, int C, int rows, int stride) {
  EncodeTiledFn enc = tensor_map_encode_fn();
  if (!enc) return set_error(FW_ERR_LAUNCH, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(stride),
                        static_cast<cuuint64_t>(rows / stride)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(C) * 2, static_cast<cuuint64_t>(C) * 2 * stride};
  cuuint32_t box[3] = {64, 1, 128};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(FW_ERR_ARG, "conv tensor map encode failed (%d)", static_cast<int>(r));
  return FW_OK;
}

template <int kSubN, int kSub, int STAGES, bool kConv>
static int launch_gemm_t(const CUtensorMap& ta, const CUtensorMap& tb, int K, int conv_c, int conv_stride,
                         const GemmEpi& ep, const void* l2_next, size_t l2_bytes, cudaStream_t s, bool pdl) {
  constexpr int BN = kSubN * kSub;
  constexpr int smem = STAGES * (128 * 64 * 2 + BN * 64 * 2) + 1024;
  auto kern = gemm_tc_kernel<kSubN, kSub, STAGES, kConv>;
  cudaError_t e = ensure_smem(kern, smem);
  if (e == cudaSuccess) {
    const int m_tiles = (ep.M + 127) / 128, n_tiles = ep.N / BN;
    const int tiles = m_tiles * n_tiles;
    const int grid = tiles < num_sms() ? tiles : num_sms();
    e = launch(kern, dim3(grid), dim3(kGemmThreads), smem, s, pdl, ta, tb, K / 64, conv_c, conv_stride, ep, m_tiles, n_tiles,
               static_cast<const char*>(l2_next), static_cast<unsigned>(l2_bytes));
  }
  return launch_status(e, "gemm_tc");
}

template <int STAGES, bool kConv>
static int launch_splitk2_t(const CUtensorMap& ta, const CUtensorMap& tb, int K, int conv_c, int conv_stride,
                            const GemmEpi& ep, const void* l2_next, size_t l2_bytes, cudaStream_t s, bool pdl) {
  constexpr int smem = STAGES * (128 * 64 * 2 + 256 * 64 * 2) + 1024;
  auto kern = gemm_splitk2_kernel<STAGES, kConv>;
  cudaError_t e = ensure_smem(kern, smem);
  if (e == cudaSuccess) {
    const int m_tiles = (ep.M + 127) / 128, tiles = m_tiles * (ep.N / 256);
    e = launch_cluster(kern, dim3(2 * tiles), dim3(kGemmThreads), smem, s, pdl, 2u, ta, tb, K / 64, conv_c,
                       conv_stride, ep, m_tiles, static_cast<const char*>(l2_next), static_cast<unsigned>(l2_bytes));
  }
  return launch_status(e, "gemm_splitk2");
}

// Long-K GEMMs whose 128 x 256 tiles, split in two along K, fit on the GPU in one round.
static bool use_splitk2(int M, int N, int K) {
  const int kb = K / 64;
  return kb >= 20 && kb % 2 == 0 && N % 256 == 0 && 2 * ((M + 127) / 128) * (N / 256) <= num_sms();
}

// Picks the N tile: the fewest tile rounds per SM, weighted by the tile width (a round costs time
// proportional to BN) and by the lower tensor efficiency of narrow tiles. The 320-wide tile has a
// single TMEM accumulator (its epilogue cannot overlap a next tile), so it is used only when every
// CTA gets exactly one tile.
static int pick_bn(int M, int N) {
  const int mt = (M + 127) / 128, sms = num_sms();
  static const int kBn[4] = {320, 256, 128, 64};
  static const float kEff[4] = {1.0f, 1.0f, 0.85f, 0.7f};
  int best = 64;
  float best_cost = 1e30f;
  for (int i = 0; i < 4; ++i) {
    if (N % kBn[i]) continue;
    const int tiles = mt * (N / kBn[i]);
    const int rounds = (tiles + sms - 1) / sms;
    if (kBn[i] == 320 && rounds > 1) continue;
    const float cost = rounds * kBn[i] / kEff[i];
    if (cost < best_cost) {
      best_cost = cost;
      best = kBn[i];
    }
  }
  return best;
}

static int gemm_dispatch(const CUtensorMap& ta, const void* B, int64_t ldb, int K, int conv_c, int conv_stride,
                         bool conv, const GemmEpi& ep, const void* l2_next, size_t l2_bytes, cudaStream_t s,
                         bool pdl) {
  if (use_splitk2(ep.M, ep.N, K)) {
    CUtensorMap tb;
    int rc = make_map_2d(&tb, B, static_cast<uint64_t>(K), static_cast<uint64_t>(ep.N), static_cast<uint64_t>(ldb), 256);
    if (rc) return rc;
    return conv ? launch_splitk2_t<4, true>(ta, tb, K, conv_c, conv_stride, ep, l2_next, l2_bytes, s, pdl)
                : launch_splitk2_t<4, false>(ta, tb, K, 0, 1, ep, l2_next, l2_bytes, s, pdl);
  }
  const int bn = pick_bn(ep.M, ep.N);
  CUtensorMap tb;
  int rc = make_map_2d(&tb, B, static_cast<uint64_t>(K), static_cast<uint64_t>(ep.N), static_cast<uint64_t>(ldb),
                       bn == 320 ? 160 : bn);
  if (rc) return rc;
  if (conv) {
    switch (bn) {
      case 320: return launch_gemm_t<160, 2, 4, true>(ta, tb, K, conv_c, conv_stride, ep, l2_next, l2_bytes, s, pdl);
      case 256: return launch_gemm_t<256, 1, 4, true>(ta, tb, K, conv_c, conv_stride, ep, l2_next, l2_bytes, s, pdl);
      case 128: return launch_gemm_t<128, 1, 6, true>(ta, tb, K, conv_c, conv_stride, ep, l2_next, l2_bytes, s, pdl);
      default: return launch_gemm_t<64, 1, 8, true>(ta, tb, K, conv_c, conv_stride, ep, l2_next, l2_bytes, s, pdl);
    }
  }
  switch (bn) {
    case 320: return launch_gemm_t<160, 2, 4, false>(ta, tb, K, 0, 1, ep, l2_next, l2_bytes, s, pdl);
    case 256: return launch_gemm_t<256, 1, 4, false>(ta, tb, K, 0, 1, ep, l2_next, l2_bytes, s, pdl);
    case 128: return launch_gemm_t<128, 1, 6, false>(ta, tb, K, 0, 1, ep, l2_next, l2_bytes, s, pdl);
    default: return launch_gemm_t<64, 1, 8, false>(ta, tb, K, 0, 1, ep, l2_next, l2_bytes, s, pdl);
  }
}

static int check_epi(const GemmEpi& ep, int K) {
  FW_REQUIRE(ep.C != nullptr, FW_ERR_NULL, "gemm: C is required");
  FW_REQUIRE(ep.M > 0 && ep.N > 0 && ep.N % 64 == 0 && K > 0 && K % 64 == 0, FW_ERR_SHAPE,
             "gemm: need M > 0, N %% 64 == 0, K %% 64 == 0 (M=%d N=%d K=%d)", ep.M, ep.N, K);
  FW_REQUIRE(ep.mode >= FW_EPI_BIAS && ep.mode <= FW_EPI_QKV_VT, FW_ERR_ARG, "gemm: unknown epilogue %d", ep.mode);
  FW_REQUIRE((ep.mode != FW_EPI_BIAS_RESID && ep.mode != FW_EPI_GELU_POS && ep.mode != FW_EPI_QKV_VT) || ep.R != nullptr,
             FW_ERR_NULL, "gemm: this epilogue needs R");
  FW_REQUIRE(ep.mode != FW_EPI_QKV_VT || (ep.N % 48 == 0 && ep.vt_col == ep.N / 3 * 2 && ep.ldr >= ep.M), FW_ERR_SHAPE,
             "gemm: FW_EPI_QKV_VT needs N %% 48 == 0 and ldr >= M");
  FW_REQUIRE(ep.mode == FW_EPI_CROSS_KV || (ep.ldc >= ep.N && ep.ldc % 8 == 0), FW_ERR_SHAPE,
             "gemm: ldc must be >= N and a multiple of 8");
  FW_REQUIRE(aligned16(ep.C) && (ep.bias == nullptr || aligned16(ep.bias)) && (ep.R == nullptr || aligned16(ep.R)),
             FW_ERR_ALIGN, "gemm: C, bias and R must be 16-byte aligned");
  FW_REQUIRE(ep.R == nullptr || ep.ldr % 8 == 0, FW_ERR_ALIGN, "gemm: ldr must be a multiple of 8");
  return FW_OK;
}

static int run_gemm(const void* A, int64_t lda, const void* B, int64_t ldb, int K, const GemmEpi& ep, cudaStream_t s,
                    bool pdl, const void* l2_next = nullptr, size_t l2_bytes = 0) {
  int rc = check_epi(ep, K);
  if (rc) return rc;
  FW_REQUIRE(A && B, FW_ERR_NULL, "gemm: A and B are required");
  FW_REQUIRE(aligned16(A) && aligned16(B) && lda % 8 == 0 && ldb % 8 == 0 && lda >= K && ldb >= K, FW_ERR_ALIGN,
             "gemm: A, B 16-byte aligned, lda/ldb >= K and multiples of 8");
  CUtensorMap ta;
  rc = make_map_2d(&ta, A, static_cast<uint64_t>(K), static_cast<uint64_t>(ep.M), static_cast<uint64_t>(lda), 128);
  if (rc) return rc;
  return gemm_dispatch(ta, B, ldb, K, 0, 1, false, ep, l2_next, l2_bytes, s, pdl);
}

static int run_conv(const void* X, int C, int rows_padded, int stride, const void* W, const GemmEpi& ep,
                    cudaStream_t s, bool pdl, const void* l2_next = nullptr, size_t l2_bytes = 0) {
  const int K = 3 * C;
  int rc = check_epi(ep, K);
  if (rc) return rc;
  FW_REQUIRE(X && W, FW_ERR_NULL, "conv: X and W are required");
  FW_REQUIRE(C % 64 == 0 && (stride == 1 || stride == 2) && rows_padded % stride == 0, FW_ERR_SHAPE,
             "conv: C %% 64 == 0, stride 1 or 2, rows divisible by stride");
  FW_REQUIRE(stride * (ep.M - 1) + 2 < rows_padded, FW_ERR_SHAPE, "conv: input too short for M output rows");
  FW_REQUIRE(aligned16(X) && aligned16(W), FW_ERR_ALIGN, "conv: X and W must be 16-byte aligned");
  CUtensorMap ta;
  rc = make_map_conv(&ta, X, C, rows_padded, stride);
  if (rc) return rc;
  return gemm_dispatch(ta, W, K, K, C, stride, true, ep, l2_next, l2_bytes, s, pdl);
}

static int run_layernorm(const void* x, const void* g, const void* b, void* y, int rows, int cols, float eps,
                         cudaStream_t s, bool pdl) {
  FW_REQUIRE(x && g && b && y, FW_ERR_NULL, "layernorm_rows: all pointers are required");
  FW_REQUIRE(rows > 0 && cols > 0 && cols % 256 == 0 && cols <= 2048, FW_ERR_SHAPE,
             "layernorm_rows: cols must be a multiple of 256, <= 2048");
  cudaError_t e = launch(layernorm_rows_kernel, dim3((rows + 7) / 8), dim3(256), 0, s, pdl,
                         static_cast<const half*>(x), static_cast<const half*>(g), static_cast<const half*>(b),
                         static_cast<half*>(y), rows, cols, eps);
  return launch_status(e, "layernorm_rows");
}

// Attention over q at columns h*64 and k at kcol + h*64 of qkv [seq, ld], and V^T [heads*64, ldv].
static int run_attention(const void* qkv, int64_t ld, int kcol, const void* vt, int64_t ldv, void* out, int seq,
                         int heads, cudaStream_t s, bool pdl) {
  FW_REQUIRE(qkv && vt && out, FW_ERR_NULL, "encoder_attention: qkv, vt and out are required");
  FW_REQUIRE(seq > 0 && heads > 0 && ld % 8 == 0 && kcol % 8 == 0 && kcol >= heads * 64 &&
                 ld >= kcol + heads * 64 && ldv % 8 == 0 && ldv >= seq,
             FW_ERR_SHAPE, "encoder_attention: bad sizes");
  FW_REQUIRE(aligned16(qkv) && aligned16(vt) && aligned16(out), FW_ERR_ALIGN,
             "encoder_attention: 16-byte alignment required");
  CUtensorMap tqk, tvt;
  int rc = make_map_2d(&tqk, qkv, static_cast<uint64_t>(kcol + heads * 64), static_cast<uint64_t>(seq),
                       static_cast<uint64_t>(ld), 64);
  if (rc) return rc;
  rc = make_map_2d(&tvt, vt, static_cast<uint64_t>(seq), static_cast<uint64_t>(heads * 64), static_cast<uint64_t>(ldv),
                   64);
  if (rc) return rc;
  cudaError_t e = ensure_smem(enc_attn_tc_kernel, kAttnSmem);
  if (e == cudaSuccess)
    e = launch(enc_attn_tc_kernel, dim3((seq + kAttnQ - 1) / kAttnQ, heads), dim3(kAttnThreads), kAttnSmem, s, pdl,
               tqk, tvt, kcol, static_cast<half*>(out), heads * 64, seq);
  return launch_status(e, "encoder_attention");
}

unsigned int read_encoder_errors(bool clear) {
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

int fw_gemm_f16(const void* A, int64_t lda, const void* B, int64_t ldb, const void* bias, void* C, int64_t ldc,
                const void* R, int64_t ldr, int M, int N, int K, int epilogue, float scale, int scale_cols,
                fw_stream_t stream) {
  GemmEpi ep{static_cast<const half*>(bias), static_cast<half*>(C), ldc, static_cast<const half*>(R), ldr, M, N,
             epilogue, scale, scale_cols, epilogue == FW_EPI_QKV_VT ? N / 3 * 2 : 0};
  return run_gemm(A, lda, B, ldb, K, ep, static_cast<cudaStream_t>(stream), false);
}

int fw_conv1d_k3_f16(const void* X, int C, int rows_padded, int stride, const void* W, const void* bias, void* Out,
                     int64_t ldc, const void* R, int64_t ldr, int M, int N, int epilogue, fw_stream_t stream) {
  GemmEpi ep{static_cast<const half*>(bias), static_cast<half*>(Out), ldc, static_cast<const half*>(R), ldr, M, N,
             epilogue, 1.f, 0};
  return run_conv(X, C, rows_padded, stride, W, ep, static_cast<cudaStream_t>(stream), false);
}

int fw_layernorm_rows(const void* x, const void* g, const void* b, void* y, int rows, int cols, float eps,
                      fw_stream_t stream) {
  return run_layernorm(x, g, b, y, rows, cols, eps, static_cast<cudaStream_t>(stream), false);
}

int fw_encoder_attention(const void* qkv, int64_t ld, int kcol, int vcol, void* out, int seq, int heads,
                         void* vt_scratch, fw_stream_t stream) {
  FW_REQUIRE(qkv && out && vt_scratch, FW_ERR_NULL, "encoder_attention: qkv, out and vt_scratch are required");
  FW_REQUIRE(seq > 0 && heads > 0 && vcol % 8 == 0 && ld >= vcol + heads * 64, FW_ERR_SHAPE,
             "encoder_attention: bad sizes");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t ldv = (seq + 7) / 8 * 8;
  cudaError_t e = launch(transpose_v_kernel, dim3((seq + 31) / 32, heads * 2), dim3(32, 8), 0, s, false,
                         static_cast<const half*>(qkv), ld, vcol, static_cast<half*>(vt_scratch), ldv, seq, heads * 64);
  int rc = launch_status(e, "encoder_attention_transpose");
  if (rc) return rc;
  return run_attention(qkv, ld, kcol, vt_scratch, ldv, out, seq, heads, s, false);
}

int fw_encoder_forward(const fw_encoder_t* e, fw_stream_t stream) {
  FW_REQUIRE(e != nullptr, FW_ERR_NULL, "encoder_forward: descriptor is NULL");
  FW_REQUIRE(e->n_layers >= 0 && e->n_layers <= FW_MAX_ENC_LAYERS && e->heads * 64 == kHidden &&
                 e->n_frames == 2 * e->n_pos && e->n_dec_layers > 0,
             FW_ERR_SHAPE, "encoder_forward: bad sizes");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int T = e->n_pos, F = e->n_frames;
  half* conv1_out = static_cast<half*>(e->conv1_out);
  half* x = static_cast<half*>(e->x);
  half* y = static_cast<half*>(e->y);
  half* qkv = static_cast<half*>(e->qkv);
  half* attn = static_cast<half*>(e->attn);
  half* ffn = static_cast<half*>(e->ffn);
  half* vt = static_cast<half*>(e->vt);
  const int64_t ldv = (T + 7) / 8 * 8;
  FW_REQUIRE(vt != nullptr, FW_ERR_NULL, "encoder_forward: vt is required");
  int rc;
  // conv1 + GELU -> rows 1..F of conv1_out (rows 0 and F+1 stay zero)
  GemmEpi ep{static_cast<const half*>(e->conv1_b), conv1_out + kHidden, kHidden, nullptr, 0, F, kHidden,
             FW_EPI_BIAS_GELU, 1.f, 0};
  if ((rc = run_conv(e->mel, 128, F + 2, 1, e->conv1_w, ep, s, true))) return rc;
  // conv2 (stride 2) + GELU + sinusoid positions -> x
  ep = GemmEpi{static_cast<const half*>(e->conv2_b), x, kHidden, static_cast<const half*>(e->pos), kHidden, T, kHidden,
               FW_EPI_GELU_POS, 1.f, 0};
  // Each GEMM warms L2 with the weights of the next GEMM in the layer sequence (qkv -> out -> fc1 ->
  // fc2 -> next layer's qkv), so their tile loads hit L2 instead of waiting on HBM.
  const size_t kSq = size_t(kHidden) * kHidden * 2, kFf = size_t(kFfn) * kHidden * 2;
  if ((rc = run_conv(conv1_out, kHidden, F + 2, 2, e->conv2_w, ep, s, true,
                     e->n_layers > 0 ? e->layers[0].qkv_w : nullptr, 3 * kSq)))
    return rc;
  for (int l = 0; l < e->n_layers; ++l) {
    const fw_encoder_layer_t& L = e->layers[l];
    const void* next_qkv = l + 1 < e->n_layers ? e->layers[l + 1].qkv_w : nullptr;
    if ((rc = run_layernorm(x, L.ln1_g, L.ln1_b, y, T, kHidden, e->eps, s, true))) return rc;
    ep = GemmEpi{static_cast<const half*>(L.qkv_b), qkv, 3 * kHidden, vt, ldv, T, 3 * kHidden,
                 FW_EPI_QKV_VT, 0.125f, kHidden, 2 * kHidden};
    if ((rc = run_gemm(y, kHidden, L.qkv_w, kHidden, kHidden, ep, s, true, L.out_w, kSq))) return rc;
    if ((rc = run_attention(qkv, 3 * kHidden, kHidden, vt, ldv, attn, T, e->heads, s, true))) return rc;
    ep = GemmEpi{static_cast<const half*>(L.out_b), x, kHidden, x, kHidden, T, kHidden, FW_EPI_BIAS_RESID, 1.f, 0};
    if ((rc = run_gemm(attn, kHidden, L.out_w, kHidden, kHidden, ep, s, true, L.fc1_w, kFf))) return rc;
    if ((rc = run_layernorm(x, L.ln2_g, L.ln2_b, y, T, kHidden, e->eps, s, true))) return rc;
    ep = GemmEpi{static_cast<const half*>(L.fc1_b), ffn, kFfn, nullptr, 0, T, kFfn, FW_EPI_BIAS_GELU, 1.f, 0};
    if ((rc = run_gemm(y, kHidden, L.fc1_w, kHidden, kHidden, ep, s, true, L.fc2_w, kFf))) return rc;
    ep = GemmEpi{static_cast<const half*>(L.fc2_b), x, kHidden, x, kHidden, T, kHidden, FW_EPI_BIAS_RESID, 1.f, 0};
    if ((rc = run_gemm(ffn, kFfn, L.fc2_w, kFfn, kFfn, ep, s, true, next_qkv, 3 * kSq))) return rc;
  }
  if ((rc = run_layernorm(x, e->final_g, e->final_b, e->enc_out, T, kHidden, e->eps, s, true))) return rc;
  const int ncross = e->n_dec_layers * 2 * kHidden;
  ep = GemmEpi{static_cast<const half*>(e->cross_b), static_cast<half*>(e->cross_kv), 0, nullptr, 0, T, ncross,
               FW_EPI_CROSS_KV, 1.f, 0};
  return run_gemm(e->enc_out, kHidden, e->cross_w, kHidden, kHidden, ep, s, true);
}

}  // extern "C"
