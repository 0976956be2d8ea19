// Device-side range coder and frequency-table quantisers (sm_100a).
//
// Coder semantics follow the reference batched coder (paths relative to the
// reference project root): encode_kernel / finalize_kernel /
// init_dec_kernel / decode_step_kernel in gpu_range_coder.py:88-210 — u64
// lower/range, u32 output words, carry resolved through a pending run of
// "inverted" words, 64-bit divide on decode, zero words past the stream end.
// PRECISION is a runtime parameter here (the reference fixes 24,
// gpu_range_coder.py:40).
//
// Two quantisers:
//   * ref  : the reference float quantiser build_cdf_fast
//            (gpu_range_coder.py:57-79) — fp32 probabilities, double
//            sequential sums.  Serial by construction; one thread per stream.
//   * bq   : this build's integer quantiser for fp32 logits, computed by one
//            warp per stream: max -> deterministic exp (Cody-Waite split +
//            degree-7 Taylor series of 2^r, explicit fmaf) -> 23-bit fixed
//            point weights -> frequencies 1 + floor(w*M/2^32) with
//            M = floor((2^P-K)*2^32/W) -> remainder on the first argmax ->
//            warp-shuffle prefix sum.  Every step after the exp is integer,
//            and the exp uses only correctly rounded operations, so a CPU
//            restatement reproduces the tables bit for bit.
#pragma once
#include <cstdint>

namespace boa {

struct RcEnc {               // 32 bytes, one per stream
  unsigned long long lower;
  unsigned long long range;
  uint32_t first_inv;        // first word of a pending (carry-undecided) run
  int32_t inv_count;         // length of that run, 0 = none
  int32_t nwords;            // words written so far
  int32_t pad;
};

struct RcDec {               // 32 bytes, one per stream
  unsigned long long lower;
  unsigned long long range;
  unsigned long long point;
  int32_t nread;
  int32_t pad;
};

enum : uint32_t {
  RC_ERR_OVERFLOW = 1u,      // a stream needed more words than its pitch
  RC_ERR_SYMBOL = 2u,        // symbol outside [0, K)
  RC_ERR_TIMEOUT = 4u,       // a bounded device wait gave up
  RC_ERR_RANGE = 8u,         // a model activation outside the operand kind's range (2xFP16: |v| >= 65504 or NaN)
};

__device__ __forceinline__ void rc_enc_reset(RcEnc& s) {
  s.lower = 0ull; s.range = ~0ull; s.first_inv = 0u; s.inv_count = 0; s.nwords = 0; s.pad = 0;
}

__device__ __forceinline__ void rc_emit(RcEnc& s, uint32_t* out, int pitch, uint32_t w,
                                        uint32_t* err) {
  if (s.nwords < pitch) {
    out[s.nwords] = w;
    s.nwords += 1;
  } else {
    atomicOr(err, RC_ERR_OVERFLOW);
  }
}

__device__ __forceinline__ void rc_flush_run(RcEnc& s, uint32_t* out, int pitch, bool carry,
                                             uint32_t* err) {
  rc_emit(s, out, pitch, carry ? s.first_inv + 1u : s.first_inv, err);
  const uint32_t fill = carry ? 0u : 0xFFFFFFFFu;
  for (int i = 1; i < s.inv_count; ++i) rc_emit(s, out, pitch, fill, err);
  s.inv_count = 0;
}

// Code one symbol with cumulative frequency `left` and frequency `freq`.
__device__ __forceinline__ void rc_enc_put(RcEnc& s, uint32_t left, uint32_t freq, int precision,
                                           uint32_t* out, int pitch, uint32_t* err) {
  const unsigned long long scale = s.range >> precision;
  const unsigned long long before = s.lower;
  s.range = scale * (unsigned long long)freq;
  s.lower = before + scale * (unsigned long long)left;      // wraps on carry
  if (s.inv_count > 0 && s.lower + s.range > s.lower) rc_flush_run(s, out, pitch, s.lower < before, err);
  while (s.range < (1ull << 32)) {
    const uint32_t top = (uint32_t)(s.lower >> 32);
    s.lower <<= 32;
    s.range <<= 32;
    if (s.inv_count > 0) {
      if (s.inv_count < 0x7FFFFFFF) s.inv_count += 1;
    } else if (s.lower + s.range > s.lower) {
      rc_emit(s, out, pitch, top, err);
    } else {
      s.inv_count = 1;
      s.first_inv = top;
    }
  }
}

__device__ __forceinline__ int rc_enc_finish(RcEnc& s, uint32_t* out, int pitch, uint32_t* err) {
  if (s.range == ~0ull) return 0;                             // nothing was coded
  const unsigned long long point = s.lower + ((1ull << 32) - 1ull);
  if (s.inv_count > 0) rc_flush_run(s, out, pitch, point < s.lower, err);
  const uint32_t pw = (uint32_t)(point >> 32);
  rc_emit(s, out, pitch, pw, err);
  const uint32_t uw = (uint32_t)((s.lower + s.range) >> 32);
  if (uw == pw) rc_emit(s, out, pitch, 0u, err);
  return s.nwords;
}

__device__ __forceinline__ uint32_t rc_next_word(RcDec& d, const uint32_t* in, int n_words) {
  uint32_t w = 0u;
  if (d.nread < n_words) { w = in[d.nread]; d.nread += 1; }
  return w;
}

__device__ __forceinline__ void rc_dec_reset(RcDec& d, const uint32_t* in, int n_words) {
  d.lower = 0ull; d.range = ~0ull; d.point = 0ull; d.nread = 0; d.pad = 0;
  d.point = (unsigned long long)rc_next_word(d, in, n_words) << 32;
  d.point |= (unsigned long long)rc_next_word(d, in, n_words);
}

// The decode target: (point - lower) / scale, clamped to 2^P - 1.
// floor(n / d) through a correctly rounded fp64 division and one integer
// correction step, for operands where the fp64 quotient is within one of the
// true floor (see the caller): exactly the integer quotient, at a fraction of
// the cost of the 64-bit by 64-bit integer division routine.
__device__ __forceinline__ unsigned long long udiv_f64(unsigned long long n, unsigned long long d) {
  unsigned long long q = (unsigned long long)(__ddiv_rn((double)n, (double)d));
  const unsigned long long p = q * d;
  if (p > n) --q;
  else if (n - p >= d) ++q;
  return q;
}

__device__ __forceinline__ uint32_t rc_dec_target(const RcDec& d, int precision,
                                                  unsigned long long& scale) {
  scale = d.range >> precision;
  const unsigned long long num = d.point - d.lower;
  // num < range < 2^64; with precision <= 16 the scale is >= 2^16, so the fp64
  // rounding of num (<= 2^11) moves the quotient by less than one
  unsigned long long q = precision <= 16 && num < (1ull << 63) ? udiv_f64(num, scale) : num / scale;
  const unsigned long long top = (1ull << precision) - 1ull;
  if (q > top) q = top;
  return (uint32_t)q;
}

__device__ __forceinline__ void rc_dec_advance(RcDec& d, unsigned long long scale, uint32_t left,
                                               uint32_t freq, const uint32_t* in, int n_words) {
  d.lower += scale * (unsigned long long)left;
  d.range = scale * (unsigned long long)freq;
  while (d.range < (1ull << 32)) {
    d.lower <<= 32;
    d.range <<= 32;
    d.point = (d.point << 32) | (unsigned long long)rc_next_word(d, in, n_words);
  }
}

// ---------------------------------------------------------------------------
// Deterministic exp(x) for x <= 0: t = x*log2(e) (fp32), k = rint(t), r = t-k,
// 2^r by the degree-7 Taylor polynomial of e^(r ln 2), result * 2^k.
// Coefficients are (ln 2)^i / i! rounded to fp32.  Only correctly rounded
// operations are used, so the CPU oracle reproduces every bit.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bq_exp(float x) {
  if (!(x > -32.0f)) return 0.0f;
  x = fminf(x, 0.0f);
  const float t = __fmul_rn(x, 0x1.715476p+0f);
  const float k = rintf(t);
  const float r = __fsub_rn(t, k);
  float p = 0x1.ffcbfcp-17f;
  p = __fmaf_rn(p, r, 0x1.430912p-13f);
  p = __fmaf_rn(p, r, 0x1.5d87fep-10f);
  p = __fmaf_rn(p, r, 0x1.3b2ab6p-7f);
  p = __fmaf_rn(p, r, 0x1.c6b08ep-5f);
  p = __fmaf_rn(p, r, 0x1.ebfbe0p-3f);
  p = __fmaf_rn(p, r, 0x1.62e430p-1f);
  p = __fmaf_rn(p, r, 1.0f);
  const int ki = (int)k;                                       // in [-47, 0]
  return __fmul_rn(p, __int_as_float((ki + 127) << 23));
}

// Warp-cooperative BQ quantiser.  Lane j owns entries [j*Q, j*Q+Q) of a row of
// K <= 32*Q logits (entries >= K are absent).  On return, f[q] holds the
// frequency of entry j*Q+q (0 for absent entries) and `base` the cumulative
// frequency of entry j*Q (exclusive prefix over lanes).  Total is 2^precision.
template <int Q>
__device__ __forceinline__ void bq_quantise_warp(const float (&v)[Q], int K, int precision, int lane,
                                                 uint32_t (&f)[Q], uint32_t& base) {
  const unsigned FULL = 0xffffffffu;
  float m = -INFINITY;
  bool bad = false;
#pragma unroll
  for (int q = 0; q < Q; ++q) {
    const int idx = lane * Q + q;
    if (idx < K) {
      if (isnan(v[q])) bad = true;
      else m = fmaxf(m, v[q]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(FULL, m, o));
  bad = __any_sync(FULL, bad);
  const uint32_t total = 1u << precision;
  if (bad || isinf(m)) {
    const uint32_t b = total / (uint32_t)K;
    const uint32_t rem = total - b * (uint32_t)K;
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      const int idx = lane * Q + q;
      f[q] = idx < K ? b + (idx == 0 ? rem : 0u) : 0u;
    }
  } else {
    uint32_t w[Q];
    uint32_t wsum = 0;
    int amax = 0x7fffffff;
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      const int idx = lane * Q + q;
      uint32_t wi = 0u;
      if (idx < K) {
        const float e = bq_exp(__fsub_rn(v[q], m));
        wi = __float2uint_rz(__fmul_rn(e, 8388608.0f));
        if (wi == 8388608u && idx < amax) amax = idx;
      }
      w[q] = wi;
      wsum += wi;
    }
    unsigned long long W = wsum;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) W += __shfl_xor_sync(FULL, W, o);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = min(amax, __shfl_xor_sync(FULL, amax, o));
    const unsigned long long freew = (unsigned long long)(total - (uint32_t)K);
    // (freew << 32) < 2^56 and W >= 2^23 (the maximum entry weighs 2^23), so
    // the fp64 quotient is within one of the floor and udiv_f64's correction
    // returns exactly the integer quotient
    const unsigned long long M = udiv_f64(freew << 32, W);
    uint32_t fsum = 0;
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      const int idx = lane * Q + q;
      f[q] = idx < K ? 1u + (uint32_t)(((unsigned long long)w[q] * M) >> 32) : 0u;
      fsum += f[q];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) fsum += __shfl_xor_sync(FULL, fsum, o);
#pragma unroll
    for (int q = 0; q < Q; ++q)
      if (lane * Q + q == amax) f[q] += total - fsum;
  }
  // exclusive prefix over lanes of the per-lane totals (fixed Kogge-Stone order)
  uint32_t mine = 0;
#pragma unroll
  for (int q = 0; q < Q; ++q) mine += f[q];
  uint32_t incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(FULL, incl, o);
    if (lane >= o) incl += y;
  }
  base = incl - mine;
}

// Given a BQ row held by the warp, return (left, freq) of symbol `sym` on every lane.
template <int Q>
__device__ __forceinline__ void bq_lookup_warp(const uint32_t (&f)[Q], uint32_t base, int sym, int lane,
                                               uint32_t& left, uint32_t& freq) {
  const int owner = sym / Q;
  uint32_t l = base, fr = 0;
#pragma unroll
  for (int q = 0; q < Q; ++q) {
    if (q < sym - owner * Q) l += f[q];
    if (q == sym - owner * Q) fr = f[q];
  }
  left = __shfl_sync(0xffffffffu, l, owner & 31);
  freq = __shfl_sync(0xffffffffu, fr, owner & 31);
}

// Find the symbol whose interval holds `target` (every lane gets the answer).
// Warp ballot over lane bases picks the owning lane; that lane scans its Q entries.
template <int Q>
__device__ __forceinline__ int bq_search_warp(const uint32_t (&f)[Q], uint32_t base, uint32_t target,
                                              int lane, uint32_t& left, uint32_t& freq) {
  uint32_t mine = 0;
#pragma unroll
  for (int q = 0; q < Q; ++q) mine += f[q];
  // a lane owns target if base <= target < base + mine (lanes with mine == 0 own nothing)
  const bool owns = (mine > 0u) && (base <= target) && (target - base < mine);
  const unsigned bal = __ballot_sync(0xffffffffu, owns);
  const int owner = bal ? (__ffs(bal) - 1) : 31;
  int s = 0;
  uint32_t l = base, fr = 0;
  bool found = false;
#pragma unroll
  for (int q = 0; q < Q; ++q) {
    if (!found && f[q] > 0u && target - l < f[q]) { s = lane * Q + q; fr = f[q]; found = true; }
    if (!found) l += f[q];
  }
  s = __shfl_sync(0xffffffffu, s, owner);
  left = __shfl_sync(0xffffffffu, l, owner);
  freq = __shfl_sync(0xffffffffu, fr, owner);
  return s;
}

// ---------------------------------------------------------------------------
// Reference float quantiser (gpu_range_coder.py:57-79), evaluated lazily:
// cumulative edge i is (u32)(run_i * scale) + i with run_i the double
// sequential sum of probs[0..i).  Serial, one thread per stream.
// ---------------------------------------------------------------------------
struct RefCdf {
  double scale;
  uint32_t step;             // degenerate rows: equal steps
  bool degenerate;
};

__device__ __forceinline__ RefCdf ref_cdf_setup(const float* probs, int K, int precision) {
  RefCdf c;
  const uint32_t total = 1u << precision;
  const uint32_t free_w = total - (uint32_t)K;
  double norm = 0.0;
  for (int i = 0; i < K; ++i) norm = __dadd_rn(norm, (double)probs[i]);
  c.degenerate = !(norm > 0.0) || !isfinite(norm);
  c.step = free_w / (uint32_t)K + 1u;
  c.scale = c.degenerate ? 0.0 : __ddiv_rn((double)free_w, norm);
  return c;
}

// Edges cdf[s] and cdf[s+1] for a known symbol.
__device__ __forceinline__ void ref_cdf_pair(const float* probs, int K, int precision, const RefCdf& c,
                                             int s, uint32_t& lo, uint32_t& hi) {
  const uint32_t total = 1u << precision;
  if (c.degenerate) {
    lo = c.step * (uint32_t)s;
    hi = (s + 1 == K) ? total : c.step * (uint32_t)(s + 1);
    return;
  }
  double run = 0.0;
  for (int i = 0; i < s; ++i) run = __dadd_rn(run, (double)probs[i]);
  lo = __double2uint_rz(__dmul_rn(run, c.scale)) + (uint32_t)s;
  if (s + 1 == K) {
    hi = total;
  } else {
    run = __dadd_rn(run, (double)probs[s]);
    hi = __double2uint_rz(__dmul_rn(run, c.scale)) + (uint32_t)(s + 1);
  }
}

// Largest s with cdf[s] <= target (the reference's linear search), plus its edges.
__device__ __forceinline__ int ref_cdf_search(const float* probs, int K, int precision, const RefCdf& c,
                                              uint32_t target, uint32_t& lo, uint32_t& hi) {
  const uint32_t total = 1u << precision;
  uint32_t prev = 0u;                       // cdf[0]
  double run = 0.0;
  int s = 0;
  for (; s < K; ++s) {
    uint32_t next;
    if (s + 1 == K) {
      next = total;
    } else if (c.degenerate) {
      next = c.step * (uint32_t)(s + 1);
    } else {
      run = __dadd_rn(run, (double)probs[s]);
      next = __double2uint_rz(__dmul_rn(run, c.scale)) + (uint32_t)(s + 1);
    }
    if (next > target) { lo = prev; hi = next; return s; }
    prev = next;
  }
  lo = prev; hi = total;
  return K - 1;
}

}  // namespace boa
