/*
 * CPU oracle for the BoaConstrictor range coder and frequency-table quantisers.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load this library, and only as the checker
 * (or the timed CPU baseline).  The product path never links or calls it.
 *
 * What it restates (paths are relative to the reference project root):
 *   - orc_cdf_ref      : build_cdf_fast, gpu_range_coder.py:57-79
 *                        (fp32 probabilities -> u32 CDF, double sequential sums,
 *                        every frequency >= 1, total 2^P)
 *   - orc_enc_*        : encode_kernel / finalize_kernel, gpu_range_coder.py:88-168
 *                        (u64 lower/range, u32 words, carry handled by the
 *                        "inverted" run of pending words)
 *   - orc_dec_*        : init_dec_kernel / decode_step_kernel,
 *                        gpu_range_coder.py:170-210 (64-bit divide, clamp,
 *                        linear CDF search, zero words past the end)
 *   - orc_cdf_bq       : the integer quantiser this build defines (no
 *                        counterpart in the reference): logits -> deterministic
 *                        exp -> 23-bit fixed point weights -> frequencies with
 *                        total 2^P, minimum 1, remainder on the first argmax.
 * The reference fixes PRECISION = 24 (gpu_range_coder.py:40); here the
 * precision is a parameter so the same core also serves PRECISION = 16.
 *
 * Build: gcc -O2 -fPIC -shared -ffp-contract=off -o oracle/liborc.so oracle/rc_oracle.c -lm
 * -ffp-contract=off matters: the quantisers must not fuse a*b+c behind our back.
 */
#include <stdint.h>
#include <string.h>
#include <math.h>

#define ORC_OK 0
#define ORC_ERR_ARGS 1
#define ORC_ERR_OVERFLOW 2

/* ------------------------------------------------------------------------- */
/* Reference float quantiser (gpu_range_coder.py:57-79).                      */
/* ------------------------------------------------------------------------- */
int orc_cdf_ref(const float* probs, int K, int precision, uint32_t* cdf)
{
    const uint32_t total = (uint32_t)1u << precision;
    if (K <= 0) { cdf[0] = 0; cdf[1] = total; return ORC_OK; }
    const uint32_t free_weight = total - (uint32_t)K;
    double norm = 0.0;
    for (int i = 0; i < K; ++i) norm += (double)probs[i];
    if (!(norm > 0.0) || !isfinite(norm)) {
        /* degenerate row: equal steps of free/K + 1, last edge pinned to total */
        uint32_t step = free_weight / (uint32_t)K + 1u;
        for (int i = 0; i < K; ++i) cdf[i] = step * (uint32_t)i;
        cdf[K] = total;
        return ORC_OK;
    }
    const double scale = (double)free_weight / norm;
    double run = 0.0;
    for (int i = 0; i < K; ++i) {
        double prod = run * scale;
        cdf[i] = (uint32_t)prod + (uint32_t)i;
        run += (double)probs[i];
    }
    cdf[K] = total;
    return ORC_OK;
}

/* ------------------------------------------------------------------------- */
/* Deterministic exp for x <= 0 (this build's spec, identical on CPU and GPU). */
/*   e^x = 2^k * 2^r with t = x*log2(e) rounded to fp32, k = rint(t), r = t-k  */
/*   2^r from the degree-7 Taylor series of e^(r ln 2), Horner with fmaf.      */
/* Coefficients are (ln 2)^i / i! rounded to fp32.                             */
/* ------------------------------------------------------------------------- */
static const float ORC_LOG2E = 0x1.715476p+0f;
static const float ORC_C[8] = {
    0x1.000000p+0f, 0x1.62e430p-1f, 0x1.ebfbe0p-3f, 0x1.c6b08ep-5f,
    0x1.3b2ab6p-7f, 0x1.5d87fep-10f, 0x1.430912p-13f, 0x1.ffcbfcp-17f };

float orc_exp_det(float x)
{
    if (!(x > -32.0f)) return 0.0f;          /* also catches -inf and NaN */
    if (x > 0.0f) x = 0.0f;                  /* inputs are logit - max <= 0 */
    float t = x * ORC_LOG2E;
    float k = rintf(t);
    float r = t - k;
    float p = ORC_C[7];
    for (int i = 6; i >= 0; --i) p = fmaf(p, r, ORC_C[i]);
    int ki = (int)k;                          /* in [-47, 0] */
    uint32_t bits = (uint32_t)(ki + 127) << 23;
    float two_k; memcpy(&two_k, &bits, 4);
    return p * two_k;
}

/* ------------------------------------------------------------------------- */
/* Integer quantiser "BQ": logits -> frequencies (total 2^P, each >= 1).       */
/* ------------------------------------------------------------------------- */
int orc_freq_bq(const float* logits, int K, int precision, uint32_t* freq)
{
    if (K <= 0 || K > 1024 || precision < 11 || precision > 24) return ORC_ERR_ARGS;
    const uint32_t total = (uint32_t)1u << precision;
    if ((uint32_t)K * 2u > total) return ORC_ERR_ARGS;
    float m = -INFINITY;
    int bad = 0;
    for (int i = 0; i < K; ++i) {
        float v = logits[i];
        if (isnan(v)) bad = 1;
        else if (v > m) m = v;
    }
    if (bad || !isfinite(m)) {
        /* non-finite row: uniform weights */
        uint32_t base = total / (uint32_t)K;
        uint32_t rem = total - base * (uint32_t)K;
        for (int i = 0; i < K; ++i) freq[i] = base;
        freq[0] += rem;
        return ORC_OK;
    }
    uint32_t w[1024];
    uint64_t W = 0;
    int amax = -1;
    for (int i = 0; i < K; ++i) {
        float e = orc_exp_det(logits[i] - m);
        uint32_t wi = (uint32_t)(e * 8388608.0f);   /* exact scale by 2^23, truncate */
        w[i] = wi;
        W += wi;
        if (amax < 0 && wi == 8388608u) amax = i;
    }
    const uint64_t free_w = (uint64_t)(total - (uint32_t)K);
    const uint64_t M = (free_w << 32) / W;
    uint32_t sum = 0;
    for (int i = 0; i < K; ++i) {
        uint32_t f = 1u + (uint32_t)(((uint64_t)w[i] * M) >> 32);
        freq[i] = f;
        sum += f;
    }
    freq[amax] += total - sum;
    return ORC_OK;
}

int orc_cdf_bq(const float* logits, int K, int precision, uint32_t* cdf)
{
    uint32_t f[1024];
    int rc = orc_freq_bq(logits, K, precision, f);
    if (rc) return rc;
    cdf[0] = 0;
    for (int i = 0; i < K; ++i) cdf[i + 1] = cdf[i] + f[i];
    return ORC_OK;
}

/* ------------------------------------------------------------------------- */
/* Range encoder (gpu_range_coder.py:88-168).                                  */
/* ------------------------------------------------------------------------- */
typedef struct {
    uint64_t lower;
    uint64_t range;
    uint32_t first_inv;     /* first word of a pending (carry-undecided) run */
    int32_t  inv_count;     /* length of the pending run, 0 = none           */
    int32_t  nwords;        /* words written so far                          */
    int32_t  overflow;      /* set if a write would pass the pitch            */
} orc_enc_t;

typedef struct {
    uint64_t lower;
    uint64_t range;
    uint64_t point;
    int32_t  nread;
    int32_t  pad;
} orc_dec_t;

void orc_enc_init(orc_enc_t* s)
{
    s->lower = 0; s->range = ~(uint64_t)0; s->first_inv = 0; s->inv_count = 0;
    s->nwords = 0; s->overflow = 0;
}

static void orc_emit(orc_enc_t* s, uint32_t* out, int pitch, uint32_t w)
{
    if (s->nwords >= pitch) { s->overflow = 1; return; }
    out[s->nwords++] = w;
}

/* Flush a pending run: the first word gets the carry, the rest become 0 on a
 * carry and all-ones otherwise. */
static void orc_flush_run(orc_enc_t* s, uint32_t* out, int pitch, int carry)
{
    orc_emit(s, out, pitch, carry ? s->first_inv + 1u : s->first_inv);
    uint32_t fill = carry ? 0u : 0xFFFFFFFFu;
    for (int i = 1; i < s->inv_count; ++i) orc_emit(s, out, pitch, fill);
    s->inv_count = 0;
}

void orc_enc_put(orc_enc_t* s, uint32_t left, uint32_t prob, int precision,
                 uint32_t* out, int pitch)
{
    const uint64_t scale = s->range >> precision;
    const uint64_t before = s->lower;
    s->range = scale * (uint64_t)prob;
    s->lower = before + scale * (uint64_t)left;          /* may wrap: carry */
    if (s->inv_count > 0 && s->lower + s->range > s->lower)
        orc_flush_run(s, out, pitch, s->lower < before);
    while (s->range < ((uint64_t)1 << 32)) {
        uint32_t top = (uint32_t)(s->lower >> 32);
        s->lower <<= 32;
        s->range <<= 32;
        if (s->inv_count > 0) {
            if (s->inv_count < 0x7FFFFFFF) s->inv_count += 1;
        } else if (s->lower + s->range > s->lower) {
            orc_emit(s, out, pitch, top);
        } else {
            s->inv_count = 1;
            s->first_inv = top;
        }
    }
}

int orc_enc_finish(orc_enc_t* s, uint32_t* out, int pitch)
{
    if (s->range == ~(uint64_t)0) return 0;             /* nothing encoded */
    const uint64_t point = s->lower + (((uint64_t)1 << 32) - 1);
    if (s->inv_count > 0) orc_flush_run(s, out, pitch, point < s->lower);
    const uint32_t pw = (uint32_t)(point >> 32);
    orc_emit(s, out, pitch, pw);
    const uint32_t uw = (uint32_t)((s->lower + s->range) >> 32);
    if (uw == pw) orc_emit(s, out, pitch, 0u);
    return s->nwords;
}

static uint32_t orc_next_word(orc_dec_t* d, const uint32_t* in, int n_words)
{
    return (d->nread < n_words) ? in[d->nread++] : 0u;
}

void orc_dec_init(orc_dec_t* d, const uint32_t* in, int n_words)
{
    d->lower = 0; d->range = ~(uint64_t)0; d->point = 0; d->nread = 0; d->pad = 0;
    for (int i = 0; i < 2; ++i) d->point = (d->point << 32) | orc_next_word(d, in, n_words);
}

int orc_dec_get(orc_dec_t* d, const uint32_t* cdf, int K, int precision,
                const uint32_t* in, int n_words)
{
    const uint64_t scale = d->range >> precision;
    uint64_t q = (d->point - d->lower) / scale;
    const uint64_t top = ((uint64_t)1 << precision) - 1;
    if (q > top) q = top;
    const uint32_t target = (uint32_t)q;
    int s = 0;                                  /* largest s with cdf[s] <= target */
    while (s + 1 <= K && cdf[s + 1] <= target) ++s;
    if (s > K - 1) s = K - 1;
    d->lower += scale * (uint64_t)cdf[s];
    d->range = scale * (uint64_t)(cdf[s + 1] - cdf[s]);
    while (d->range < ((uint64_t)1 << 32)) {
        d->lower <<= 32;
        d->range <<= 32;
        d->point = (d->point << 32) | orc_next_word(d, in, n_words);
    }
    return s;
}

/* ------------------------------------------------------------------------- */
/* Batch drivers used by the tests and the CPU baseline.                       */
/*   mode 0: rows are fp32 probabilities, reference float quantiser            */
/*   mode 1: rows are fp32 logits, BQ integer quantiser                        */
/* rows[N][T][K], syms[N][T]; stream i codes its first counts[i] symbols.      */
/* ------------------------------------------------------------------------- */
static int orc_row_cdf(int mode, const float* row, int K, int precision, uint32_t* cdf)
{
    return mode == 0 ? orc_cdf_ref(row, K, precision, cdf) : orc_cdf_bq(row, K, precision, cdf);
}

int orc_encode_batch(int N, int T, int K, int precision, int mode,
                     const float* rows, const int32_t* syms, const int32_t* counts,
                     uint32_t* out, int pitch, int32_t* sizes)
{
    if (K <= 0 || K > 1024) return ORC_ERR_ARGS;
    uint32_t cdf[1025];
    int status = ORC_OK;
    for (int i = 0; i < N; ++i) {
        orc_enc_t s; orc_enc_init(&s);
        uint32_t* o = out + (size_t)i * (size_t)pitch;
        int n = counts[i] < T ? counts[i] : T;
        for (int t = 0; t < n; ++t) {
            int32_t sym = syms[(size_t)i * T + t];
            if (sym < 0 || sym >= K) continue;   /* reference skips such lanes */
            int rc = orc_row_cdf(mode, rows + ((size_t)i * T + t) * K, K, precision, cdf);
            if (rc) return rc;
            orc_enc_put(&s, cdf[sym], cdf[sym + 1] - cdf[sym], precision, o, pitch);
        }
        sizes[i] = orc_enc_finish(&s, o, pitch);
        if (s.overflow) status = ORC_ERR_OVERFLOW;
    }
    return status;
}

int orc_decode_batch(int N, int T, int K, int precision, int mode,
                     const float* rows, const uint32_t* in, int pitch,
                     const int32_t* sizes, const int32_t* counts, int32_t* syms_out)
{
    if (K <= 0 || K > 1024) return ORC_ERR_ARGS;
    uint32_t cdf[1025];
    for (int i = 0; i < N; ++i) {
        const uint32_t* w = in + (size_t)i * (size_t)pitch;
        orc_dec_t d; orc_dec_init(&d, w, sizes[i]);
        int n = counts[i] < T ? counts[i] : T;
        for (int t = 0; t < n; ++t) {
            int rc = orc_row_cdf(mode, rows + ((size_t)i * T + t) * K, K, precision, cdf);
            if (rc) return rc;
            syms_out[(size_t)i * T + t] = orc_dec_get(&d, cdf, K, precision, w, sizes[i]);
        }
    }
    return ORC_OK;
}

/* Encode with explicit per-symbol frequency tables: cdfs[N][T][K+1]. */
int orc_encode_cdfs(int N, int T, int K, int precision, const uint32_t* cdfs,
                    const int32_t* syms, const int32_t* counts,
                    uint32_t* out, int pitch, int32_t* sizes)
{
    int status = ORC_OK;
    for (int i = 0; i < N; ++i) {
        orc_enc_t s; orc_enc_init(&s);
        uint32_t* o = out + (size_t)i * (size_t)pitch;
        int n = counts[i] < T ? counts[i] : T;
        for (int t = 0; t < n; ++t) {
            const uint32_t* c = cdfs + ((size_t)i * T + t) * (size_t)(K + 1);
            int32_t sym = syms[(size_t)i * T + t];
            if (sym < 0 || sym >= K) continue;
            orc_enc_put(&s, c[sym], c[sym + 1] - c[sym], precision, o, pitch);
        }
        sizes[i] = orc_enc_finish(&s, o, pitch);
        if (s.overflow) status = ORC_ERR_OVERFLOW;
    }
    return status;
}

/* ------------------------------------------------------------------------- */
/* Step-wise drivers (one symbol per stream per call), for loops whose next   */
/* table depends on the previous decoded symbol — the shape of the            */
/* reference's CPU codec loops (codec.py:203-235, 292-320).                   */
/* ------------------------------------------------------------------------- */
size_t orc_enc_state_size(void) { return sizeof(orc_enc_t); }
size_t orc_dec_state_size(void) { return sizeof(orc_dec_t); }

void orc_enc_init_n(orc_enc_t* s, int N) { for (int i = 0; i < N; ++i) orc_enc_init(&s[i]); }

int orc_encode_step(int N, int K, int precision, int mode, const float* rows, const int32_t* syms,
                    const uint8_t* mask, orc_enc_t* st, uint32_t* out, int pitch)
{
    uint32_t cdf[1025];
    for (int i = 0; i < N; ++i) {
        if (mask && !mask[i]) continue;
        int32_t s = syms[i];
        if (s < 0 || s >= K) continue;
        int rc = orc_row_cdf(mode, rows + (size_t)i * K, K, precision, cdf);
        if (rc) return rc;
        orc_enc_put(&st[i], cdf[s], cdf[s + 1] - cdf[s], precision, out + (size_t)i * pitch, pitch);
    }
    return ORC_OK;
}

int orc_encode_finish_n(int N, orc_enc_t* st, uint32_t* out, int pitch, int32_t* sizes)
{
    int status = ORC_OK;
    for (int i = 0; i < N; ++i) {
        sizes[i] = orc_enc_finish(&st[i], out + (size_t)i * pitch, pitch);
        if (st[i].overflow) status = ORC_ERR_OVERFLOW;
    }
    return status;
}

void orc_dec_init_n(orc_dec_t* d, int N, const uint32_t* in, int pitch, const int32_t* sizes)
{
    for (int i = 0; i < N; ++i) orc_dec_init(&d[i], in + (size_t)i * pitch, sizes[i]);
}

int orc_decode_step(int N, int K, int precision, int mode, const float* rows, const uint8_t* mask,
                    orc_dec_t* d, const uint32_t* in, int pitch, const int32_t* sizes, int32_t* syms_out)
{
    uint32_t cdf[1025];
    for (int i = 0; i < N; ++i) {
        if (mask && !mask[i]) continue;
        int rc = orc_row_cdf(mode, rows + (size_t)i * K, K, precision, cdf);
        if (rc) return rc;
        syms_out[i] = orc_dec_get(&d[i], cdf, K, precision, in + (size_t)i * pitch, sizes[i]);
    }
    return ORC_OK;
}
