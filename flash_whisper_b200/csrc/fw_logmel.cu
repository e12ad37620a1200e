// GPU log-mel front end: the math of custom/model.py:93-98 (torch.stft + mel GEMM + log10 +
// per-clip max clamp + affine), itself the GPU form of WhisperFeatureExtractor's
// _torch_extract_fbank_features (transformers feature_extraction_whisper.py).
//
// Kernel 1 (power_mel): a CTA takes 16 consecutive frames of one clip, stages the reflect-padded
// samples in shared memory, applies the periodic Hann window, evaluates the 201-bin real DFT of
// each frame directly in fp32 (twiddles from a 400-entry table), forms |X|^2, projects onto the
// 128 mel filters, takes log10(max(., 1e-10)), writes fp32 to scratch (time-major) and folds the
// CTA maximum into the clip maximum with an order-preserving atomicMax.
// Kernel 2 (normalize): y = fp16((max(x, clip_max - 8) + 4) / 4) in the requested layout.
#include "fw_common.cuh"
#include "fw_host.h"

namespace fw {

FW_DEFINE_ERROR_WORD();

constexpr int kNfft = 400;
constexpr int kHop = 160;
constexpr int kBins = kNfft / 2 + 1;  // 201
constexpr int kMels = 128;
constexpr int kFramesPerCta = 16;

__device__ __forceinline__ int reflect_index(int j, int len) {
  // torch.stft(center=True, pad_mode='reflect'): pad n_fft/2 on each side by reflection
  // without repeating the edge sample.
  if (j < 0) j = -j;
  if (j >= len) j = 2 * (len - 1) - j;
  return j;
}

__global__ void __launch_bounds__(256) logmel_power_kernel(const float* __restrict__ wave, int n_samples,
                                                           int n_frames, const float* __restrict__ filters,
                                                           float* __restrict__ scratch,
                                                           unsigned int* __restrict__ clip_max) {
  __shared__ float cos_t[kNfft];
  __shared__ float sin_t[kNfft];
  __shared__ __align__(16) float frames[kFramesPerCta][kNfft];
  __shared__ float power[kFramesPerCta][kBins + 3];
  __shared__ float red[8];
  const int clip = blockIdx.y;
  const int f0 = blockIdx.x * kFramesPerCta;
  const int nf = min(kFramesPerCta, n_frames - f0);
  const float* x = wave + static_cast<size_t>(clip) * n_samples;

  for (int m = threadIdx.x; m < kNfft; m += blockDim.x) {
    double s, c;
    sincospi(2.0 * m / kNfft, &s, &c);
    cos_t[m] = static_cast<float>(c);
    sin_t[m] = static_cast<float>(s);
  }
  pdl_wait();
  pdl_trigger();
  __syncthreads();
  // Stage windowed frames: frame f covers padded samples [f*hop, f*hop + n_fft), i.e. original
  // indices f*hop - n_fft/2 + n.
  for (int i = threadIdx.x; i < kFramesPerCta * kNfft; i += blockDim.x) {
    const int f = i / kNfft, n = i - f * kNfft;
    float v = 0.f;
    if (f < nf) {
      const int j = reflect_index((f0 + f) * kHop - kNfft / 2 + n, n_samples);
      const float w = 0.5f - 0.5f * cos_t[n];  // periodic Hann
      v = x[j] * w;
    }
    frames[f][n] = v;
  }
  __syncthreads();

  // Real DFT, one bin per thread for all 16 frames.
  const int k = threadIdx.x;
  if (k < kBins) {
    float re[kFramesPerCta], im[kFramesPerCta];
#pragma unroll
    for (int f = 0; f < kFramesPerCta; ++f) re[f] = im[f] = 0.f;
    int idx = 0;  // (k * n) mod n_fft
    for (int n = 0; n < kNfft; n += 4) {
      float c4[4], s4[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        c4[j] = cos_t[idx];
        s4[j] = sin_t[idx];
        idx += k;
        if (idx >= kNfft) idx -= kNfft;
      }
#pragma unroll
      for (int f = 0; f < kFramesPerCta; ++f) {
        const float4 xv = *reinterpret_cast<const float4*>(&frames[f][n]);
        re[f] = fmaf(xv.x, c4[0], re[f]);
        im[f] = fmaf(-xv.x, s4[0], im[f]);
        re[f] = fmaf(xv.y, c4[1], re[f]);
        im[f] = fmaf(-xv.y, s4[1], im[f]);
        re[f] = fmaf(xv.z, c4[2], re[f]);
        im[f] = fmaf(-xv.z, s4[2], im[f]);
        re[f] = fmaf(xv.w, c4[3], re[f]);
        im[f] = fmaf(-xv.w, s4[3], im[f]);
      }
    }
#pragma unroll
    for (int f = 0; f < kFramesPerCta; ++f) power[f][k] = fmaf(re[f], re[f], im[f] * im[f]);
  }
  __syncthreads();

  // Mel projection + log10, scratch is [clip][frame][mel] (coalesced along mel).
  float local_max = -INFINITY;
  for (int i = threadIdx.x; i < nf * kMels; i += blockDim.x) {
    const int f = i / kMels, m = i - f * kMels;
    float s = 0.f;
    for (int b = 0; b < kBins; ++b) s = fmaf(__ldg(filters + b * kMels + m), power[f][b], s);
    const float lv = log10f(fmaxf(s, 1e-10f));
    scratch[(static_cast<size_t>(clip) * n_frames + f0 + f) * kMels + m] = lv;
    local_max = fmaxf(local_max, lv);
  }
  local_max = warp_max(local_max);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = local_max;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = red[0];
    for (int i = 1; i < 8; ++i) m = fmaxf(m, red[i]);
    atomicMax(clip_max + clip, float_to_ordered(m));
  }
}

// layout 0: out[clip][mel][frame]; layout 1: out[clip][frame + 1][mel] with zero rows 0 and
// n_frames + 1. A CTA handles 32 frames x 128 mels, transposing through shared memory for layout 0.
__global__ void __launch_bounds__(256) logmel_norm_kernel(const float* __restrict__ scratch,
                                                          const unsigned int* __restrict__ clip_max, int n_frames,
                                                          half* __restrict__ out, int layout) {
  __shared__ float tile[32][kMels + 1];
  pdl_wait();
  pdl_trigger();
  const int clip = blockIdx.y;
  const int f0 = blockIdx.x * 32;
  const float lo = ordered_to_float(clip_max[clip]) - 8.0f;
  const float* src = scratch + static_cast<size_t>(clip) * n_frames * kMels;
  if (layout == 1) {
    half* dst = out + static_cast<size_t>(clip) * (n_frames + 2) * kMels;
    for (int i = threadIdx.x; i < 32 * kMels; i += blockDim.x) {
      const int f = f0 + i / kMels, m = i % kMels;
      if (f < n_frames) {
        const float v = fmaxf(src[static_cast<size_t>(f) * kMels + m], lo);
        dst[static_cast<size_t>(f + 1) * kMels + m] = __float2half((v + 4.0f) / 4.0f);
      }
    }
    if (blockIdx.x == 0 && threadIdx.x < kMels) {
      dst[threadIdx.x] = __float2half(0.f);
      dst[static_cast<size_t>(n_frames + 1) * kMels + threadIdx.x] = __float2half(0.f);
    }
    return;
  }
  for (int i = threadIdx.x; i < 32 * kMels; i += blockDim.x) {
    const int f = i / kMels, m = i % kMels;
    tile[f][m] = (f0 + f < n_frames) ? src[static_cast<size_t>(f0 + f) * kMels + m] : 0.f;
  }
  __syncthreads();
  half* dst = out + static_cast<size_t>(clip) * kMels * n_frames;
  for (int i = threadIdx.x; i < 32 * kMels; i += blockDim.x) {
    const int m = i / 32, f = i % 32;
    if (f0 + f < n_frames) {
      const float v = fmaxf(tile[f][m], lo);
      dst[static_cast<size_t>(m) * n_frames + f0 + f] = __float2half((v + 4.0f) / 4.0f);
    }
  }
}

unsigned int read_logmel_errors(bool clear) {
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

extern "C" int fw_log_mel(const float* wave, int batch, int n_samples, const float* filters, float* scratch,
                          unsigned int* clip_max, void* mel_out, int layout, fw_stream_t stream) {
  FW_REQUIRE(wave && filters && scratch && clip_max && mel_out, FW_ERR_NULL, "log_mel: all pointers are required");
  FW_REQUIRE(batch > 0 && n_samples >= kNfft && n_samples % kHop == 0, FW_ERR_SHAPE,
             "log_mel: n_samples must be a positive multiple of %d and >= %d", kHop, kNfft);
  FW_REQUIRE(layout == 0 || layout == 1, FW_ERR_ARG, "log_mel: layout must be 0 or 1");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int n_frames = n_samples / kHop;
  cudaError_t e = cudaMemsetAsync(clip_max, 0, sizeof(unsigned int) * batch, s);
  if (e == cudaSuccess)
    e = launch(logmel_power_kernel, dim3((n_frames + kFramesPerCta - 1) / kFramesPerCta, batch), dim3(256), 0, s,
               false, wave, n_samples, n_frames, filters, scratch, clip_max);
  int rc = launch_status(e, "log_mel power");
  if (rc) return rc;
  e = launch(logmel_norm_kernel, dim3((n_frames + 31) / 32, batch), dim3(256), 0, s, true,
             static_cast<const float*>(scratch), static_cast<const unsigned int*>(clip_max), n_frames,
             static_cast<half*>(mel_out), layout);
  return launch_status(e, "log_mel normalize");
}
