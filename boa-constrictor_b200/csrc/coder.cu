// Batched range coder kernels and their C-ABI (libboa_b200.so).
//
// Replaces the reference's embedded pybind11 extension RangeCoderBatch
// (gpu_range_coder.py:212-324).  Differences by design:
//   * stream-ordered: every entry point takes a cudaStream_t and never
//     synchronises the device (the reference calls cudaDeviceSynchronize after
//     each launch, gpu_range_coder.py:271,276,296,304);
//   * the BQ quantiser path runs one warp per stream with coalesced 32-byte
//     loads per lane and a warp-ballot symbol search on decode;
//   * output overflow / bad symbols raise a device error flag that the host
//     reports, instead of writing past the pitch.
#include <cuda_runtime.h>
#include <cstdint>
#include <cstring>
#include <cstdio>
#include <string>
#include <vector>

#include "rc_device.cuh"
#include "boa_b200.h"
#include "capi_util.h"

namespace boa {

// ------------------------------- kernels -----------------------------------

__global__ void k_rc_reset_enc(RcEnc* enc, int32_t* sizes, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) { rc_enc_reset(enc[i]); sizes[i] = 0; }
}

// BQ encode: one warp per stream, Q logits per lane.
template <int Q>
__global__ void __launch_bounds__(256) k_rc_encode_bq(int n, int K, int precision, const float* __restrict__ logits,
                                                      const int32_t* __restrict__ syms, const uint8_t* __restrict__ mask,
                                                      RcEnc* __restrict__ enc, uint32_t* __restrict__ words, int pitch,
                                                      uint32_t* err) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < n; i += warps) {
    if (mask && mask[i] == 0) continue;
    const int s = syms[i];
    if (s < 0 || s >= K) {
      if (lane == 0) atomicOr(err, RC_ERR_SYMBOL);
      continue;
    }
    float v[Q];
    const float* row = logits + (size_t)i * (size_t)K;
    if (Q % 4 == 0 && K == 32 * Q) {
#pragma unroll
      for (int q = 0; q < Q; q += 4) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(row + lane * Q + q));
        v[q] = t.x; v[q + 1] = t.y; v[q + 2] = t.z; v[q + 3] = t.w;
      }
    } else {
#pragma unroll
      for (int q = 0; q < Q; ++q) {
        const int idx = lane * Q + q;
        v[q] = idx < K ? __ldg(row + idx) : 0.0f;
      }
    }
    uint32_t f[Q], base;
    bq_quantise_warp<Q>(v, K, precision, lane, f, base);
    uint32_t left, freq;
    bq_lookup_warp<Q>(f, base, s, lane, left, freq);
    if (lane == 0) {
      RcEnc st = enc[i];
      rc_enc_put(st, left, freq, precision, words + (size_t)i * (size_t)pitch, pitch, err);
      enc[i] = st;
    }
  }
}

// Reference-quantiser encode: one thread per stream (the float quantiser is a
// serial double chain, gpu_range_coder.py:57-79).
__global__ void __launch_bounds__(128) k_rc_encode_ref(int n, int K, int precision, const float* __restrict__ probs,
                                                       const int32_t* __restrict__ syms, const uint8_t* __restrict__ mask,
                                                       RcEnc* __restrict__ enc, uint32_t* __restrict__ words, int pitch,
                                                       uint32_t* err) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  if (mask && mask[i] == 0) return;
  const int s = syms[i];
  if (s < 0 || s >= K) { atomicOr(err, RC_ERR_SYMBOL); return; }
  const float* row = probs + (size_t)i * (size_t)K;
  const RefCdf c = ref_cdf_setup(row, K, precision);
  uint32_t lo, hi;
  ref_cdf_pair(row, K, precision, c, s, lo, hi);
  RcEnc st = enc[i];
  rc_enc_put(st, lo, hi - lo, precision, words + (size_t)i * (size_t)pitch, pitch, err);
  enc[i] = st;
}

__global__ void k_rc_finalize(int n, RcEnc* enc, uint32_t* words, int pitch, int32_t* sizes, uint32_t* err) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  RcEnc st = enc[i];
  sizes[i] = rc_enc_finish(st, words + (size_t)i * (size_t)pitch, pitch, err);
  enc[i] = st;
}

__global__ void k_rc_init_dec(int n, const uint32_t* words, int pitch, const int32_t* sizes, RcDec* dec) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  int nw = sizes[i];
  nw = nw < 0 ? 0 : (nw > pitch ? pitch : nw);
  RcDec d;
  rc_dec_reset(d, words + (size_t)i * (size_t)pitch, nw);
  dec[i] = d;
}

template <int Q>
__global__ void __launch_bounds__(256) k_rc_decode_bq(int n, int K, int precision, const float* __restrict__ logits,
                                                      const uint8_t* __restrict__ mask, RcDec* __restrict__ dec,
                                                      const uint32_t* __restrict__ words, int pitch,
                                                      const int32_t* __restrict__ sizes, int32_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < n; i += warps) {
    if (mask && mask[i] == 0) continue;
    float v[Q];
    const float* row = logits + (size_t)i * (size_t)K;
    if (Q % 4 == 0 && K == 32 * Q) {
#pragma unroll
      for (int q = 0; q < Q; q += 4) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(row + lane * Q + q));
        v[q] = t.x; v[q + 1] = t.y; v[q + 2] = t.z; v[q + 3] = t.w;
      }
    } else {
#pragma unroll
      for (int q = 0; q < Q; ++q) {
        const int idx = lane * Q + q;
        v[q] = idx < K ? __ldg(row + idx) : 0.0f;
      }
    }
    uint32_t f[Q], base;
    bq_quantise_warp<Q>(v, K, precision, lane, f, base);
    RcDec d = dec[i];
    unsigned long long scale;
    const uint32_t target = rc_dec_target(d, precision, scale);
    uint32_t left, freq;
    const int s = bq_search_warp<Q>(f, base, target, lane, left, freq);
    if (lane == 0) {
      int nw = sizes[i];
      nw = nw < 0 ? 0 : (nw > pitch ? pitch : nw);
      rc_dec_advance(d, scale, left, freq, words + (size_t)i * (size_t)pitch, nw);
      dec[i] = d;
      out[i] = s;
    }
  }
}


// Multi-step BQ coder: one warp per stream codes n_steps symbols in one
// launch, the coder state in registers of lane 0 and the next step's logits
// row loaded while the current one is coded.  Step t reads row / symbol / mask
// slot (t % period) (period <= 0: slot t) at the given per-slot strides.
template <int Q>
__device__ __forceinline__ void rc_load_row(float (&v)[Q], const float* __restrict__ row, int K, int lane) {
  if (Q % 4 == 0 && K == 32 * Q) {
#pragma unroll
    for (int q = 0; q < Q; q += 4) {
      const float4 t = __ldg(reinterpret_cast<const float4*>(row + lane * Q + q));
      v[q] = t.x; v[q + 1] = t.y; v[q + 2] = t.z; v[q + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      const int idx = lane * Q + q;
      v[q] = idx < K ? __ldg(row + idx) : 0.0f;
    }
  }
}

template <int Q>
__global__ void __launch_bounds__(256) k_rc_encode_bq_steps(int n, int K, int precision, int n_steps, int period,
                                                            const float* __restrict__ logits, long long row_stride,
                                                            const int32_t* __restrict__ syms, long long sym_stride,
                                                            const uint8_t* __restrict__ mask, long long mask_stride,
                                                            RcEnc* __restrict__ enc, uint32_t* __restrict__ words,
                                                            int pitch, uint32_t* err) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < n; i += warps) {
    RcEnc st = enc[i];
    uint32_t* wrow = words + (size_t)i * (size_t)pitch;
    float v[Q];
    rc_load_row<Q>(v, logits + (size_t)i * (size_t)K, K, lane);
    int slot = 0;
    for (int t = 0; t < n_steps; ++t) {
      const int next = (period > 0 && slot + 1 == period) ? 0 : slot + 1;
      float nv[Q];
      if (t + 1 < n_steps) rc_load_row<Q>(nv, logits + (long long)next * row_stride + (size_t)i * (size_t)K, K, lane);
      const bool on = !mask || mask[(long long)slot * mask_stride + i] != 0;
      const int s = syms[(long long)slot * sym_stride + i];
      if (on && (s < 0 || s >= K)) {
        if (lane == 0) atomicOr(err, RC_ERR_SYMBOL);
      } else if (on) {
        uint32_t f[Q], base;
        bq_quantise_warp<Q>(v, K, precision, lane, f, base);
        uint32_t left, freq;
        bq_lookup_warp<Q>(f, base, s, lane, left, freq);
        if (lane == 0) rc_enc_put(st, left, freq, precision, wrow, pitch, err);
      }
      if (t + 1 < n_steps) {
#pragma unroll
        for (int q = 0; q < Q; ++q) v[q] = nv[q];
      }
      slot = next;
    }
    if (lane == 0) enc[i] = st;
  }
}

template <int Q>
__global__ void __launch_bounds__(256) k_rc_decode_bq_steps(int n, int K, int precision, int n_steps, int period,
                                                            const float* __restrict__ logits, long long row_stride,
                                                            const uint8_t* __restrict__ mask, long long mask_stride,
                                                            RcDec* __restrict__ dec, const uint32_t* __restrict__ words,
                                                            int pitch, const int32_t* __restrict__ sizes,
                                                            int32_t* __restrict__ out, long long out_stride) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < n; i += warps) {
    RcDec d = dec[i];
    const uint32_t* wrow = words + (size_t)i * (size_t)pitch;
    int nw = sizes[i];
    nw = nw < 0 ? 0 : (nw > pitch ? pitch : nw);
    float v[Q];
    rc_load_row<Q>(v, logits + (size_t)i * (size_t)K, K, lane);
    int slot = 0;
    for (int t = 0; t < n_steps; ++t) {
      const int next = (period > 0 && slot + 1 == period) ? 0 : slot + 1;
      float nv[Q];
      if (t + 1 < n_steps) rc_load_row<Q>(nv, logits + (long long)next * row_stride + (size_t)i * (size_t)K, K, lane);
      if (!mask || mask[(long long)slot * mask_stride + i] != 0) {
        uint32_t f[Q], base;
        bq_quantise_warp<Q>(v, K, precision, lane, f, base);
        unsigned long long scale;
        const uint32_t target = rc_dec_target(d, precision, scale);
        uint32_t left, freq;
        const int s = bq_search_warp<Q>(f, base, target, lane, left, freq);
        rc_dec_advance(d, scale, left, freq, wrow, nw);     // every lane: the state stays warp-uniform
        if (lane == 0) out[(long long)slot * out_stride + i] = s;
      }
      if (t + 1 < n_steps) {
#pragma unroll
        for (int q = 0; q < Q; ++q) v[q] = nv[q];
      }
      slot = next;
    }
    if (lane == 0) dec[i] = d;
  }
}

__global__ void __launch_bounds__(128) k_rc_decode_ref(int n, int K, int precision, const float* __restrict__ probs,
                                                       const uint8_t* __restrict__ mask, RcDec* __restrict__ dec,
                                                       const uint32_t* __restrict__ words, int pitch,
                                                       const int32_t* __restrict__ sizes, int32_t* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  if (mask && mask[i] == 0) return;
  const float* row = probs + (size_t)i * (size_t)K;
  const RefCdf c = ref_cdf_setup(row, K, precision);
  RcDec d = dec[i];
  unsigned long long scale;
  const uint32_t target = rc_dec_target(d, precision, scale);
  uint32_t lo, hi;
  const int s = ref_cdf_search(row, K, precision, c, target, lo, hi);
  int nw = sizes[i];
  nw = nw < 0 ? 0 : (nw > pitch ? pitch : nw);
  rc_dec_advance(d, scale, lo, hi - lo, words + (size_t)i * (size_t)pitch, nw);
  dec[i] = d;
  out[i] = s;
}

}  // namespace boa

// ------------------------------- C-ABI -------------------------------------
using namespace boa;

struct boa_rc_batch {
  int n, K, pitch, precision, quantiser, device;
  RcEnc* enc = nullptr;
  RcDec* dec = nullptr;
  uint32_t* words = nullptr;
  int32_t* sizes = nullptr;
  uint32_t* err = nullptr;
};

static int rc_grid_warps(int n) {
  // one warp per stream, 8 warps per block, grid a multiple of the SM count
  int blocks = (n + 7) / 8;
  const int cap = 148 * 16;
  return blocks < cap ? (blocks < 1 ? 1 : blocks) : cap;
}

// The BQ kernels load each row of K = 256 or 1024 logits as float4 (Q % 4 == 0
// and K == 32 * Q): those rows must start on 16-byte boundaries.  Checked on
// the host so a misaligned pointer is an argument error, not a device fault.
static int bq_rows_aligned(int K, const float* rows, int64_t row_stride, const char* who) {
  if (K != 256 && K != 1024) return BOA_OK;
  if ((reinterpret_cast<uintptr_t>(rows) & 15u) != 0 || (row_stride & 3) != 0)
    return boa_fail(BOA_ERR_ARG, std::string(who) + ": with K = 256 or 1024 the logits rows (and the per-step "
                                                    "stride) must be 16-byte aligned");
  return BOA_OK;
}

extern "C" {

BOA_API int boa_rc_create(boa_rc_batch** out, int n_streams, int k_symbols, int pitch_words,
                          int precision, int quantiser, int device) {
  if (!out) return boa_fail(BOA_ERR_ARG, "boa_rc_create: null out");
  *out = nullptr;
  if (n_streams < 1) return boa_fail(BOA_ERR_ARG, "boa_rc_create: n_streams must be >= 1");
  if (k_symbols < 1 || k_symbols > 1024) return boa_fail(BOA_ERR_ARG, "boa_rc_create: K must be in [1, 1024]");
  if (pitch_words < 1) return boa_fail(BOA_ERR_ARG, "boa_rc_create: pitch_words must be >= 1");
  if (precision < 11 || precision > 24) return boa_fail(BOA_ERR_ARG, "boa_rc_create: precision must be in [11, 24]");
  if ((2 * k_symbols) > (1 << precision)) return boa_fail(BOA_ERR_ARG, "boa_rc_create: K too large for precision");
  if (quantiser != BOA_QUANT_REF && quantiser != BOA_QUANT_BQ)
    return boa_fail(BOA_ERR_ARG, "boa_rc_create: unknown quantiser");
  BOA_CUDA(cudaSetDevice(device));
  boa_rc_batch* b = new boa_rc_batch();
  b->n = n_streams; b->K = k_symbols; b->pitch = pitch_words; b->precision = precision;
  b->quantiser = quantiser; b->device = device;
  const size_t wbytes = (size_t)n_streams * (size_t)pitch_words * sizeof(uint32_t);
  cudaError_t e = cudaMalloc(&b->enc, sizeof(RcEnc) * (size_t)n_streams);
  if (e == cudaSuccess) e = cudaMalloc(&b->dec, sizeof(RcDec) * (size_t)n_streams);
  if (e == cudaSuccess) e = cudaMalloc(&b->words, wbytes);
  if (e == cudaSuccess) e = cudaMalloc(&b->sizes, sizeof(int32_t) * (size_t)n_streams);
  if (e == cudaSuccess) e = cudaMalloc(&b->err, sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMemset(b->words, 0, wbytes);
  if (e == cudaSuccess) e = cudaMemset(b->err, 0, sizeof(uint32_t));
  if (e == cudaSuccess) {
    k_rc_reset_enc<<<(n_streams + 255) / 256, 256>>>(b->enc, b->sizes, n_streams);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    boa_rc_destroy(b);
    return boa_fail(BOA_ERR_CUDA, std::string("boa_rc_create: ") + cudaGetErrorString(e));
  }
  *out = b;
  return BOA_OK;
}

BOA_API int boa_rc_destroy(boa_rc_batch* b) {
  if (!b) return BOA_OK;
  cudaSetDevice(b->device);
  cudaFree(b->enc); cudaFree(b->dec); cudaFree(b->words); cudaFree(b->sizes); cudaFree(b->err);
  delete b;
  return BOA_OK;
}

BOA_API int boa_rc_info(const boa_rc_batch* b, int* n_streams, int* k_symbols, int* pitch_words,
                        int* precision, int* quantiser) {
  if (!b) return boa_fail(BOA_ERR_ARG, "boa_rc_info: null handle");
  if (n_streams) *n_streams = b->n;
  if (k_symbols) *k_symbols = b->K;
  if (pitch_words) *pitch_words = b->pitch;
  if (precision) *precision = b->precision;
  if (quantiser) *quantiser = b->quantiser;
  return BOA_OK;
}

BOA_API int boa_rc_load(boa_rc_batch* b, const uint32_t* host_words, const int32_t* host_sizes, void* stream) {
  if (!b || !host_words || !host_sizes) return boa_fail(BOA_ERR_ARG, "boa_rc_load: null argument");
  for (int i = 0; i < b->n; ++i)
    if (host_sizes[i] < 0 || host_sizes[i] > b->pitch)
      return boa_fail(BOA_ERR_ARG, "boa_rc_load: compressed stream exceeds pitch; increase pitch");
  BOA_CUDA(cudaSetDevice(b->device));
  cudaStream_t s = (cudaStream_t)stream;
  BOA_CUDA(cudaMemcpyAsync(b->words, host_words, (size_t)b->n * (size_t)b->pitch * sizeof(uint32_t),
                           cudaMemcpyHostToDevice, s));
  BOA_CUDA(cudaMemcpyAsync(b->sizes, host_sizes, sizeof(int32_t) * (size_t)b->n, cudaMemcpyHostToDevice, s));
  BOA_CUDA(cudaStreamSynchronize(s));   // host buffers may be pageable and short-lived
  return BOA_OK;
}

BOA_API int boa_rc_set_sizes(boa_rc_batch* b, const int32_t* host_sizes, void* stream) {
  if (!b || !host_sizes) return boa_fail(BOA_ERR_ARG, "boa_rc_set_sizes: null argument");
  BOA_CUDA(cudaSetDevice(b->device));
  cudaStream_t s = (cudaStream_t)stream;
  BOA_CUDA(cudaMemcpyAsync(b->sizes, host_sizes, sizeof(int32_t) * (size_t)b->n, cudaMemcpyHostToDevice, s));
  BOA_CUDA(cudaStreamSynchronize(s));
  return BOA_OK;
}

static int rc_check_err(boa_rc_batch* b, cudaStream_t s) {
  uint32_t e = 0;
  BOA_CUDA(cudaMemcpyAsync(&e, b->err, sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
  BOA_CUDA(cudaStreamSynchronize(s));
  if (e & RC_ERR_OVERFLOW) return boa_fail(BOA_ERR_OVERFLOW, "range coder: a stream exceeded its pitch (words lost)");
  if (e & RC_ERR_SYMBOL) return boa_fail(BOA_ERR_ARG, "range coder: symbol outside [0, K)");
  return BOA_OK;
}

BOA_API int boa_rc_get_sizes(boa_rc_batch* b, int32_t* host_sizes, void* stream) {
  if (!b || !host_sizes) return boa_fail(BOA_ERR_ARG, "boa_rc_get_sizes: null argument");
  BOA_CUDA(cudaSetDevice(b->device));
  cudaStream_t s = (cudaStream_t)stream;
  BOA_CUDA(cudaMemcpyAsync(host_sizes, b->sizes, sizeof(int32_t) * (size_t)b->n, cudaMemcpyDeviceToHost, s));
  return rc_check_err(b, s);
}

BOA_API int boa_rc_get_words(boa_rc_batch* b, uint32_t* host_words, void* stream) {
  if (!b || !host_words) return boa_fail(BOA_ERR_ARG, "boa_rc_get_words: null argument");
  BOA_CUDA(cudaSetDevice(b->device));
  cudaStream_t s = (cudaStream_t)stream;
  BOA_CUDA(cudaMemcpyAsync(host_words, b->words, (size_t)b->n * (size_t)b->pitch * sizeof(uint32_t),
                           cudaMemcpyDeviceToHost, s));
  return rc_check_err(b, s);
}

BOA_API int boa_rc_device_buffers(boa_rc_batch* b, uint32_t** words, int32_t** sizes) {
  if (!b) return boa_fail(BOA_ERR_ARG, "boa_rc_device_buffers: null handle");
  if (words) *words = b->words;
  if (sizes) *sizes = b->sizes;
  return BOA_OK;
}

BOA_API int boa_rc_encode_step(boa_rc_batch* b, const int32_t* d_symbols, const float* d_rows,
                               const uint8_t* d_mask, void* stream) {
  if (!b || !d_symbols || !d_rows) return boa_fail(BOA_ERR_ARG, "boa_rc_encode_step: null argument");
  if (b->quantiser == BOA_QUANT_BQ) {
    const int rc = bq_rows_aligned(b->K, d_rows, 0, "boa_rc_encode_step");
    if (rc) return rc;
  }
  BOA_CUDA(cudaSetDevice(b->device));
  cudaStream_t s = (cudaStream_t)stream;
  if (b->quantiser == BOA_QUANT_BQ) {
    const int grid = rc_grid_warps(b->n);
    if (b->K <= 256)
      k_rc_encode_bq<8><<<grid, 256, 0, s>>>(b->n, b->K, b->precision, d_rows, d_symbols, d_mask, b->enc,
                                             b->words, b->pitch, b->err);
    else
      k_rc_encode_bq<32><<<grid, 256, 0, s>>>(b->n, b->K, b->precision, d_rows, d_symbols, d_mask, b->enc,
                                              b->words, b->pitch, b->err);
  } else {
    k_rc_encode_ref<<<(b->n + 127) / 128, 128, 0, s>>>(b->n, b->K, b->precision, d_rows, d_symbols, d_mask,
                                                       b->enc, b->words, b->pitch, b->err);
  }
  BOA_CUDA(cudaGetLastError());
  return BOA_OK;
}

BOA_API int boa_rc_finalize(boa_rc_batch* b, void* stream) {
  if (!b) return boa_fail(BOA_ERR_ARG, "boa_rc_finalize: null handle");
  BOA_CUDA(cudaSetDevice(b->device));
  k_rc_finalize<<<(b->n + 127) / 128, 128, 0, (cudaStream_t)stream>>>(b->n, b->enc, b->words, b->pitch, b->sizes,
                                                                       b->err);
  BOA_CUDA(cudaGetLastError());
  return BOA_OK;
}

BOA_API int boa_rc_init_decoder(boa_rc_batch* b, void* stream) {
  if (!b) return boa_fail(BOA_ERR_ARG, "boa_rc_init_decoder: null handle");
  BOA_CUDA(cudaSetDevice(b->device));
  k_rc_init_dec<<<(b->n + 127) / 128, 128, 0, (cudaStream_t)stream>>>(b->n, b->words, b->pitch, b->sizes, b->dec);
  BOA_CUDA(cudaGetLastError());
  return BOA_OK;
}

BOA_API int boa_rc_decode_step(boa_rc_batch* b, const float* d_rows, int32_t* d_out_symbols,
                               const uint8_t* d_mask, void* stream) {
  if (!b || !d_rows || !d_out_symbols) return boa_fail(BOA_ERR_ARG, "boa_rc_decode_step: null argument");
  if (b->quantiser == BOA_QUANT_BQ) {
    const int rc = bq_rows_aligned(b->K, d_rows, 0, "boa_rc_decode_step");
    if (rc) return rc;
  }
  BOA_CUDA(cudaSetDevice(b->device));
  cudaStream_t s = (cudaStream_t)stream;
  if (b->quantiser == BOA_QUANT_BQ) {
    const int grid = rc_grid_warps(b->n);
    if (b->K <= 256)
      k_rc_decode_bq<8><<<grid, 256, 0, s>>>(b->n, b->K, b->precision, d_rows, d_mask, b->dec, b->words,
                                             b->pitch, b->sizes, d_out_symbols);
    else
      k_rc_decode_bq<32><<<grid, 256, 0, s>>>(b->n, b->K, b->precision, d_rows, d_mask, b->dec, b->words,
                                              b->pitch, b->sizes, d_out_symbols);
  } else {
    k_rc_decode_ref<<<(b->n + 127) / 128, 128, 0, s>>>(b->n, b->K, b->precision, d_rows, d_mask, b->dec,
                                                       b->words, b->pitch, b->sizes, d_out_symbols);
  }
  BOA_CUDA(cudaGetLastError());
  return BOA_OK;
}

BOA_API int boa_rc_encode_steps(boa_rc_batch* b, int n_steps, int period, const int32_t* d_symbols,
                                int64_t sym_stride, const float* d_rows, int64_t row_stride, const uint8_t* d_mask,
                                int64_t mask_stride, void* stream) {
  if (!b || !d_symbols || !d_rows || n_steps < 0) return boa_fail(BOA_ERR_ARG, "boa_rc_encode_steps: bad argument");
  if (b->quantiser != BOA_QUANT_BQ)
    return boa_fail(BOA_ERR_UNSUPPORTED, "boa_rc_encode_steps: BOA_QUANT_BQ handles only");
  if (const int rc = bq_rows_aligned(b->K, d_rows, row_stride, "boa_rc_encode_steps")) return rc;
  if (n_steps == 0) return BOA_OK;
  BOA_CUDA(cudaSetDevice(b->device));
  cudaStream_t s = (cudaStream_t)stream;
  const int grid = rc_grid_warps(b->n);
  if (b->K <= 256)
    k_rc_encode_bq_steps<8><<<grid, 256, 0, s>>>(b->n, b->K, b->precision, n_steps, period, d_rows, row_stride,
                                                 d_symbols, sym_stride, d_mask, mask_stride, b->enc, b->words,
                                                 b->pitch, b->err);
  else
    k_rc_encode_bq_steps<32><<<grid, 256, 0, s>>>(b->n, b->K, b->precision, n_steps, period, d_rows, row_stride,
                                                  d_symbols, sym_stride, d_mask, mask_stride, b->enc, b->words,
                                                  b->pitch, b->err);
  BOA_CUDA(cudaGetLastError());
  return BOA_OK;
}

BOA_API int boa_rc_decode_steps(boa_rc_batch* b, int n_steps, int period, const float* d_rows, int64_t row_stride,
                                int32_t* d_out_symbols, int64_t out_stride, const uint8_t* d_mask,
                                int64_t mask_stride, void* stream) {
  if (!b || !d_rows || !d_out_symbols || n_steps < 0) return boa_fail(BOA_ERR_ARG, "boa_rc_decode_steps: bad argument");
  if (b->quantiser != BOA_QUANT_BQ)
    return boa_fail(BOA_ERR_UNSUPPORTED, "boa_rc_decode_steps: BOA_QUANT_BQ handles only");
  if (const int rc = bq_rows_aligned(b->K, d_rows, row_stride, "boa_rc_decode_steps")) return rc;
  if (n_steps == 0) return BOA_OK;
  BOA_CUDA(cudaSetDevice(b->device));
  cudaStream_t s = (cudaStream_t)stream;
  const int grid = rc_grid_warps(b->n);
  if (b->K <= 256)
    k_rc_decode_bq_steps<8><<<grid, 256, 0, s>>>(b->n, b->K, b->precision, n_steps, period, d_rows, row_stride,
                                                 d_mask, mask_stride, b->dec, b->words, b->pitch, b->sizes,
                                                 d_out_symbols, out_stride);
  else
    k_rc_decode_bq_steps<32><<<grid, 256, 0, s>>>(b->n, b->K, b->precision, n_steps, period, d_rows, row_stride,
                                                  d_mask, mask_stride, b->dec, b->words, b->pitch, b->sizes,
                                                  d_out_symbols, out_stride);
  BOA_CUDA(cudaGetLastError());
  return BOA_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free whole-stream encode.
//
// Some callers cannot allocate device memory when they code: a plugin host or
// framework that owns the device memory pool and forbids allocation after
// start-up, a real-time service that must not stall on cudaMalloc (which can
// synchronise the device), or code that must not fragment a memory pool it
// does not own.  boa_rc_encode_noalloc serves them: the caller passes the
// inputs and the outputs, and the per-stream coder state (the scratch that
// boa_rc_create would allocate) lives in the file-scope array below instead.
// Each call ends by copying the array's error word back to the host, so it
// synchronises the caller's stream.
//
// Limits and sharing:
//   * at most kNoAllocMaxStreams streams per call (2 MiB of state); larger
//     calls are rejected with BOA_ERR_ARG;
//   * the array is one per device and every call shares it: each call clears
//     the state of the streams it uses (and the error word) before coding, so
//     nothing from an earlier call leaks in, but two calls that overlap on the
//     GPU (different streams, different host threads) race on it and corrupt
//     each other's output;
//   * every GPU that loads this library keeps the array until process exit;
//   * the first call on a device looks up the array's device address
//     (cudaGetSymbolAddress) and caches it for the life of the process: a
//     device reset (cudaDeviceReset) invalidates the cached address and is not
//     supported while the library is loaded.
// ---------------------------------------------------------------------------
namespace boa {
constexpr int kNoAllocMaxStreams = 1 << 16;
constexpr size_t kNoAllocStateBytes = (size_t)kNoAllocMaxStreams * sizeof(RcEnc);
static __device__ __align__(256) unsigned char g_rc_noalloc_scratch[kNoAllocStateBytes + 256];
}  // namespace boa

#include <mutex>

static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[64] = {nullptr};

// Device address of the scratch array on the current device (looked up once).
static int noalloc_scratch(int device, void** out) {
  if (device < 0 || device >= 64) return boa_fail(BOA_ERR_ARG, "boa_rc_encode_noalloc: device index out of range");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, boa::g_rc_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return boa_fail(BOA_ERR_CUDA, std::string("boa_rc_encode_noalloc: cudaGetSymbolAddress: ") +
                                        cudaGetErrorString(e));
    g_noalloc_ptr[device] = p;
  }
  *out = g_noalloc_ptr[device];
  return BOA_OK;
}

__global__ void k_rc_noalloc_clear(RcEnc* enc, int n, uint32_t* err) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) rc_enc_reset(enc[i]);
  if (i == 0) *err = 0u;
}

extern "C" BOA_API int boa_rc_encode_noalloc(int n_streams, int k_symbols, int n_steps, int precision,
                                             const float* d_logits, const int32_t* d_symbols, const uint8_t* d_mask,
                                             uint32_t* d_words, int pitch_words, int32_t* d_sizes, void* stream) {
  if (n_streams < 1 || n_streams > kNoAllocMaxStreams)
    return boa_fail(BOA_ERR_ARG, "boa_rc_encode_noalloc: n_streams must be in [1, 65536] (static scratch limit)");
  if (k_symbols < 1 || k_symbols > 1024) return boa_fail(BOA_ERR_ARG, "boa_rc_encode_noalloc: K must be in [1, 1024]");
  if (n_steps < 0 || pitch_words < 1) return boa_fail(BOA_ERR_ARG, "boa_rc_encode_noalloc: bad n_steps / pitch");
  if (precision < 11 || precision > 24 || 2 * k_symbols > (1 << precision))
    return boa_fail(BOA_ERR_ARG, "boa_rc_encode_noalloc: precision out of range for K");
  if (!d_words || !d_sizes || (n_steps > 0 && (!d_logits || !d_symbols)))
    return boa_fail(BOA_ERR_ARG, "boa_rc_encode_noalloc: null argument");
  if (n_steps > 0)
    if (const int rc = bq_rows_aligned(k_symbols, d_logits, 0, "boa_rc_encode_noalloc")) return rc;
  int device = 0;
  BOA_CUDA(cudaGetDevice(&device));
  void* base = nullptr;
  int rc = noalloc_scratch(device, &base);
  if (rc) return rc;
  RcEnc* enc = reinterpret_cast<RcEnc*>(base);
  uint32_t* err = reinterpret_cast<uint32_t*>(reinterpret_cast<unsigned char*>(base) + kNoAllocStateBytes);
  cudaStream_t s = (cudaStream_t)stream;
  k_rc_noalloc_clear<<<(n_streams + 255) / 256, 256, 0, s>>>(enc, n_streams, err);
  BOA_CUDA(cudaGetLastError());
  const int grid = rc_grid_warps(n_streams);
  for (int t = 0; t < n_steps; ++t) {
    const float* rows = d_logits + (size_t)t * n_streams * k_symbols;
    const int32_t* syms = d_symbols + (size_t)t * n_streams;
    const uint8_t* mask = d_mask ? d_mask + (size_t)t * n_streams : nullptr;
    if (k_symbols <= 256)
      k_rc_encode_bq<8><<<grid, 256, 0, s>>>(n_streams, k_symbols, precision, rows, syms, mask, enc, d_words,
                                             pitch_words, err);
    else
      k_rc_encode_bq<32><<<grid, 256, 0, s>>>(n_streams, k_symbols, precision, rows, syms, mask, enc, d_words,
                                              pitch_words, err);
  }
  k_rc_finalize<<<(n_streams + 127) / 128, 128, 0, s>>>(n_streams, enc, d_words, pitch_words, d_sizes, err);
  BOA_CUDA(cudaGetLastError());
  uint32_t e = 0;
  BOA_CUDA(cudaMemcpyAsync(&e, err, sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
  BOA_CUDA(cudaStreamSynchronize(s));
  if (e & RC_ERR_OVERFLOW) return boa_fail(BOA_ERR_OVERFLOW, "boa_rc_encode_noalloc: a stream exceeded its pitch");
  if (e & RC_ERR_SYMBOL) return boa_fail(BOA_ERR_ARG, "boa_rc_encode_noalloc: symbol outside [0, K)");
  return BOA_OK;
}
