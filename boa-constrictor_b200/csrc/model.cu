// BoaConstrictor model + fused codec loop for sm_100a: host side and C-ABI.
// The kernel (k_boa_step) and its launch helpers are in model_kernel.cuh; this
// file packs the weights into the kernel's tile streams, builds the device
// model, and exposes the boa_model_* / boa_codec_* entry points.
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <climits>
#include <cstdint>
#include <cstring>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>
#include <algorithm>
#include <utility>

#include "model_kernel.cuh"

namespace boa {

constexpr int kCT = 16;                // value columns of the diagnostic GEMM

// ---------------------------------------------------------------------------
// Diagnostic single-CTA GEMM through the same pipeline pieces:
//   out[m][n] = sum_k W[m][k] * X[n][k]   (W pre-packed tiles, X via store_operand)
// With the split kind the operand has 2 * kCT rows (hi and lo halves) and each
// (M tile, K slice) is a hi tile followed by a lo tile.
// ---------------------------------------------------------------------------
template <int KIND>
__global__ void __launch_bounds__(256, 1) k_diag_gemm(const uint8_t* wtiles, const float* X, float* out, int M, int K,
                                                      uint32_t* err) {
  constexpr int HL = tc::OpKind<KIND>::kHiLo;
  constexpr int CT = kCT * HL;                       // operand rows
  constexpr int kTilesPer = HL == 1 ? 1 : 2;         // weight tiles per (M tile, K slice)
  constexpr int PER = 128 / tc::OpKind<KIND>::kElemBytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int kBbuf = CT * 1024 * tc::OpKind<KIND>::kElemBytes;   // B operand, K up to 1024
  uint8_t* tile = smem;                              // one A tile
  uint8_t* bbuf = smem + kTileBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kTileBytes + kBbuf);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 5);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_mt = M / 128, n_ks = K / PER;
  if (tid == 0) {
    tc::mbar_init(&bars[0], 1);   // tile landed
    tc::mbar_init(&bars[1], 1);   // MMAs done
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (warp == 1) { tc::tmem_alloc(tslot, 512); tc::tmem_relinquish(); }
  for (int i = tid; i < kCT * K; i += blockDim.x) tc::store_operand<KIND>(bbuf, i / K, i % K, CT, X[i]);
  tc::fence_proxy_async_smem();
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tslot;
  uint32_t ph = 0;
  for (int mt = 0; mt < n_mt; ++mt) {
    for (int ks = 0; ks < n_ks; ++ks) {
      for (int hl = 0; hl < kTilesPer; ++hl) {
        if (tid == 0) {
          tc::mbar_arrive_expect_tx(&bars[0], kTileBytes);
          tc::bulk_g2s(tile, wtiles + (((long long)mt * n_ks + ks) * kTilesPer + hl) * kTileBytes, kTileBytes,
                       &bars[0], tc::policy_evict_first());
          if (tc::mbar_wait(&bars[0], ph, abort_flag, kWaitBudget)) {
            tc::tc_fence_after();
            // kind 4: the lo' tile takes rows [2 VC, 4 VC) into columns [VC, 3 VC)
            const uint32_t row0 = (HL == 4 && hl) ? 2 * kCT * 128 : 0, dcol = (HL == 4 && hl) ? kCT : 0;
            const uint32_t a0 = tc::smem_u32(tile), b0 = tc::smem_u32(bbuf) + ks * CT * 128 + row0;
            for (int kk = 0; kk < 4; ++kk)
              tc::mma<KIND>(tmem + (uint32_t)(mt * CT) + dcol, tc::sdesc_sw128(a0 + kk * 32),
                            tc::sdesc_sw128(b0 + kk * 32), tc::idesc<KIND>(128, HL == 4 ? CT / 2 : CT),
                            (ks > 0 || hl > 0 || kk > 0) ? 1u : 0u);
            tc::mma_commit(&bars[1]);
            tc::mbar_wait(&bars[1], ph, abort_flag, kWaitBudget);   // tile buffer reusable
          }
        }
        ph ^= 1u;
        __syncthreads();
      }
    }
  }
  tc::tc_fence_after();
  if (warp < 4) {
    for (int mt = 0; mt < n_mt; ++mt) {
      float v[16];
      const uint32_t ta = tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)(mt * CT);
      if constexpr (HL == 2) {
        float w[8];
        tc::tmem_ld8_sum(ta, ta + kCT, w);
        for (int n = 0; n < 8; ++n) v[n] = w[n];
        tc::tmem_ld8_sum(ta + 8, ta + kCT + 8, w);
        for (int n = 0; n < 8; ++n) v[8 + n] = w[n];
      } else if constexpr (HL == 4) {
        float w[8];
        tc::tmem_ld8_sum_s11(ta, ta + kCT, w);
        for (int n = 0; n < 8; ++n) v[n] = w[n];
        tc::tmem_ld8_sum_s11(ta + 8, ta + kCT + 8, w);
        for (int n = 0; n < 8; ++n) v[8 + n] = w[n];
      } else {
        tc::tmem_ld16(ta, v);
      }
      const int m = mt * 128 + 32 * warp + lane;
      for (int n = 0; n < kCT; ++n) out[(long long)m * kCT + n] = v[n];
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (tid == 0 && *abort_flag) atomicOr(err, RC_ERR_TIMEOUT);
  if (warp == 1) { tc::tc_fence_after(); tc::tmem_dealloc(tmem, 512); }
}

// ------------------------------- host side ---------------------------------
static uint32_t f32_bits(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
static float bits_f32(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }

// Round-to-nearest (ties away) to tf32, as cvt.rna.tf32.f32 does.
static uint32_t to_tf32_bits(float f) {
  uint32_t u = f32_bits(f);
  if ((u & 0x7f800000u) != 0x7f800000u) u = (u + 0x1000u) & 0xffffe000u;
  return u;
}

// One M tile of a GEMM's weights: rows [mt*128, mt*128+128) of W [M_real x K]
// (row-major fp32, leading dimension ldw; rows >= M_real and columns >= K_real
// are zero).
struct MTile {
  const float* W;
  int M_real, K_real, ldw, mt;
  int ks0 = 0;       // first K slice (x_proj's second K half)
};

// Append the SW128 tile images of one GEMM's M tiles, each with n_ks K slices.
// Order: M tile by M tile, or (pairs) the K slices of M tiles 2q and 2q+1
// interleaved -- (2q, 0), (2q+1, 0), (2q, 1), ... -- which is the order in which
// the two MMA issuers of a single-CTA kernel take them.  The split kinds emit,
// for every (M tile, K slice), the tile of the weights' hi halves followed by
// the tile of their lo halves (kind 3: tf32 hi, tf32 lo; kind 4: fp16 hi,
// fp16 residual scaled by 2^11).
static void pack_gemm(std::vector<uint8_t>& out, const std::vector<MTile>& tiles, int n_ks, int kind, bool pairs) {
  const int eb = (kind == 0 || kind == 3) ? 4 : 2;
  const int per = 128 / eb;
  const int hl_n = (kind == 3 || kind == 4) ? 2 : 1;
  std::vector<std::pair<int, int>> order;   // (index into tiles, ks)
  const int n_mt = (int)tiles.size();
  for (int m0 = 0; m0 < n_mt; m0 += pairs ? 2 : 1) {
    const int nm = pairs ? std::min(2, n_mt - m0) : 1;
    for (int ks = 0; ks < n_ks; ++ks)
      for (int h = 0; h < nm; ++h) order.push_back({m0 + h, ks});
  }
  for (const auto& o : order) {
    const float* W = tiles[o.first].W;
    const int M_real = tiles[o.first].M_real, K_real = tiles[o.first].K_real, ldw = tiles[o.first].ldw;
    const int mt = tiles[o.first].mt, ks = tiles[o.first].ks0 + o.second;
    for (int hl = 0; hl < hl_n; ++hl) {
      const size_t base = out.size();
      out.resize(base + kTileBytes, 0);
      uint8_t* t = out.data() + base;
      for (int r = 0; r < 128; ++r) {
        const int m = mt * 128 + r;
        for (int e = 0; e < per; ++e) {
          const int k = ks * per + e;
          const float v = (m < M_real && k < K_real) ? W[(size_t)m * ldw + k] : 0.0f;
          const int byte = e * eb;
          const int chunk = byte >> 4;
          uint8_t* p = t + r * 128 + (((chunk ^ (r & 7)) << 4) | (byte & 15));
          if (kind == 3) {
            const uint32_t hi = to_tf32_bits(v);
            const uint32_t b = hl == 0 ? hi : to_tf32_bits(v - bits_f32(hi));
            std::memcpy(p, &b, 4);
          } else if (kind == 4) {
            const __half hi = __float2half_rn(v);
            const unsigned short h =
                hl == 0 ? __half_as_ushort(hi) : __half_as_ushort(__float2half_rn((v - __half2float(hi)) * 2048.0f));
            std::memcpy(p, &h, 2);
          } else if (kind == 0) {
            const uint32_t b = to_tf32_bits(v);
            std::memcpy(p, &b, 4);
          } else if (kind == BOA_WEIGHTS_BF16) {
            const unsigned short h = __bfloat16_as_ushort(__float2bfloat16_rn(v));
            std::memcpy(p, &h, 2);
          } else {
            const unsigned short h = __half_as_ushort(__float2half_rn(v));
            std::memcpy(p, &h, 2);
          }
        }
      }
    }
  }
}

// M tiles mt0 .. mt0+n_mt-1 of W, appended to a GEMM's tile list.
static void add_mtiles(std::vector<MTile>& v, const float* W, int M_real, int K_real, int ldw, int mt0, int n_mt) {
  for (int mt = mt0; mt < mt0 + n_mt; ++mt) v.push_back(MTile{W, M_real, K_real, ldw, mt});
}

}  // namespace boa

using namespace boa;

namespace {

// Walk the flat convert_boa_weights.py order (convert_boa_weights.py:16-135).
struct FlatReader {
  const float* p;
  size_t n, pos = 0;
  bool ok = true;
  const float* take(size_t k) {
    if (pos + k > n) { ok = false; return nullptr; }
    const float* r = p + pos;
    pos += k;
    return r;
  }
};

struct LayerW {
  const float *w_in, *w_x, *w_dt, *w_out, *w1, *w2;
};

// Pack one rank's weight stream of a `split`-way cluster in consumption order
// (single-CTA streams pair up M tiles for the two MMA issuers).
static void pack_stream(std::vector<uint8_t>& tiles, const TilePlan& p, int rank, int D, int V, int kind,
                        const std::vector<LayerW>& lw, const float* wh0, const float* wh2) {
  const int E = 2 * D, R = cdiv(D, 16), DBC = R + 32, F = 4 * D;
  const bool pairs = p.split == 1;
  auto gemm = [&](const float* W, int M_real, int K_real, int ldw, int mt0, int n_mt, int n_ks) {
    std::vector<MTile> v;
    add_mtiles(v, W, M_real, K_real, ldw, mt0, n_mt);
    pack_gemm(tiles, v, n_ks, kind, pairs);
  };
  for (const LayerW& w : lw) {
    std::vector<MTile> in;                                                   // x rows, then z rows
    add_mtiles(in, w.w_in, 2 * E, D, D, rank * p.ltE, p.ltE);
    add_mtiles(in, w.w_in, 2 * E, D, D, p.mtE + rank * p.ltE, p.ltE);
    pack_gemm(tiles, in, p.kD, kind, pairs);
    std::vector<MTile> xp;                                                   // M tile 0 as two K halves
    add_mtiles(xp, w.w_x, DBC, E, E, 0, 1);
    add_mtiles(xp, w.w_x, DBC, E, E, 0, 1);
    xp[1].ks0 = p.kE / 2;
    pack_gemm(tiles, xp, p.kE / 2, kind, pairs);
    gemm(w.w_dt, E, R, R, rank * p.ltE, p.ltE, 1);
    gemm(w.w_out, D, E, E, rank * p.ltD, p.ltD, p.kE);
    gemm(w.w1, F, D, D, rank * p.ltF, p.ltF, p.kD);
    gemm(w.w2, D, F, F, rank * p.ltD, p.ltD, p.kF);
  }
  gemm(wh0, D, D, D, rank * p.ltD, p.ltD, p.kD);
  gemm(wh2, V, D, D, rank * p.ltV, p.ltV, p.kD);
}

template <int D>
int build_model(boa_model* m, const float* flat, size_t n_floats, std::vector<uint8_t>& tiles,
                std::vector<uint8_t>& tiles2, std::vector<float>& params) {
  using LP = LayerParams<D>;
  const int E = 2 * D, R = cdiv(D, 16), DBC = R + 32, F = 4 * D, V = m->V, L = m->L, kind = m->kind;
  FlatReader fr{flat, n_floats};
  const float* emb = fr.take((size_t)V * D);
  params.assign((size_t)LP::stride * L + D + 256 + (size_t)V * D, 0.0f);
  std::vector<LayerW> lw(L);
  for (int l = 0; l < L; ++l) {
    float* lp = params.data() + (size_t)LP::stride * l;
    const float* ln1w = fr.take(D); const float* ln1b = fr.take(D);
    const float* w_in = fr.take((size_t)2 * E * D); fr.take((size_t)2 * E);      // in_proj.bias slot (zeros)
    const float* convw = fr.take((size_t)E * 4); const float* convb = fr.take(E);
    const float* w_x = fr.take((size_t)DBC * E);
    const float* w_dt = fr.take((size_t)E * R); const float* b_dt = fr.take(E);
    const float* A_log = fr.take((size_t)E * 16); const float* Dv = fr.take(E);
    const float* w_out = fr.take((size_t)D * E); fr.take(D);                     // out_proj.bias slot (zeros)
    const float* ln2w = fr.take(D); const float* ln2b = fr.take(D);
    const float* w1 = fr.take((size_t)F * D); const float* b1 = fr.take(F);
    const float* w2 = fr.take((size_t)D * F); const float* b2 = fr.take(D);
    if (!fr.ok) return boa_fail(BOA_ERR_ARG, "boa_model_create: flat weight vector too short for the config");
    std::memcpy(lp + LP::ln1w, ln1w, D * 4); std::memcpy(lp + LP::ln1b, ln1b, D * 4);
    std::memcpy(lp + LP::convw, convw, (size_t)E * 16); std::memcpy(lp + LP::convb, convb, E * 4);
    std::memcpy(lp + LP::dtb, b_dt, E * 4); std::memcpy(lp + LP::Dp, Dv, E * 4);
    for (int i = 0; i < E * 16; ++i)   // A*log2(e) with A = -exp(A_log), for exp2 in the scan
      lp[LP::A2 + i] = (float)(-std::exp((double)A_log[i]) * 1.4426950408889634);
    std::memcpy(lp + LP::ln2w, ln2w, D * 4); std::memcpy(lp + LP::ln2b, ln2b, D * 4);
    std::memcpy(lp + LP::b1, b1, F * 4); std::memcpy(lp + LP::b2, b2, D * 4);
    lw[l] = LayerW{w_in, w_x, w_dt, w_out, w1, w2};
  }
  const float* wh0 = fr.take((size_t)D * D); const float* bh0 = fr.take(D);
  const float* wh2 = fr.take((size_t)V * D); const float* bh2 = fr.take(V);
  if (!fr.ok) return boa_fail(BOA_ERR_ARG, "boa_model_create: flat weight vector too short for the config");
  if (fr.pos != n_floats) return boa_fail(BOA_ERR_ARG, "boa_model_create: flat weight vector longer than the config");
  float* g = params.data() + (size_t)LP::stride * L;
  std::memcpy(g, bh0, D * 4);
  std::memcpy(g + D, bh2, V * 4);
  std::memcpy(g + D + 256, emb, (size_t)V * D * 4);
  pack_stream(tiles, m->plan, 0, D, V, kind, lw, wh0, wh2);
  if (tiles.size() != (size_t)m->plan.per_step * kTileBytes)
    return boa_fail(BOA_ERR_ARG, "boa_model_create: internal tile count mismatch");
  if (m->has_split2) {
    pack_stream(tiles2, m->plan2, 0, D, V, kind, lw, wh0, wh2);
    pack_stream(tiles2, m->plan2, 1, D, V, kind, lw, wh0, wh2);
    if (tiles2.size() != (size_t)2 * m->plan2.per_step * kTileBytes)
      return boa_fail(BOA_ERR_ARG, "boa_model_create: internal tile count mismatch (split)");
  }
  return BOA_OK;
}

size_t conv_state_bytes(const boa_model* m, int n) { return (size_t)n * m->L * (2 * m->D) * 16; }
size_t ssm_state_bytes(const boa_model* m, int n) { return (size_t)n * m->L * (2 * m->D) * 64; }

#ifdef BOA_PHASE_PROFILE
// BOA_PHASE_PROFILE=1: time the phases of CTA 0 and print them (SM cycles) to stderr.
int launch_step_profiled(const boa_model* m, StepArgs& a, int n_chunks, cudaStream_t s);
#endif

int launch_step(const boa_model* m, StepArgs& a, int n_chunks, cudaStream_t s) {
#ifdef BOA_PHASE_PROFILE
  const char* pe = getenv("BOA_PHASE_PROFILE");
  if (pe && pe[0] == '1' && a.prof == nullptr) return launch_step_profiled(m, a, n_chunks, s);
#endif
  a.n_layers = m->L;
  a.vocab = m->V;
  a.params = m->d_params;
  a.err = m->d_err;
  const int positions = a.mode == MODE_LOGITS ? a.n_steps : a.pos1 - a.pos0;
  switch (m->D * 8 + m->kind) {
    case 64 * 8 + 0: return launch_step_t<64, 0>(m, a, n_chunks, s, positions);
    case 64 * 8 + 1: return launch_step_t<64, 1>(m, a, n_chunks, s, positions);
    case 64 * 8 + 2: return launch_step_t<64, 2>(m, a, n_chunks, s, positions);
    case 64 * 8 + 3: return launch_step_t<64, 3>(m, a, n_chunks, s, positions);
    case 64 * 8 + 4: return launch_step_t<64, 4>(m, a, n_chunks, s, positions);
    case 256 * 8 + 0: return launch_step_t<256, 0>(m, a, n_chunks, s, positions);
    case 256 * 8 + 1: return launch_step_t<256, 1>(m, a, n_chunks, s, positions);
    case 256 * 8 + 2: return launch_step_t<256, 2>(m, a, n_chunks, s, positions);
    case 256 * 8 + 3: return launch_step_t<256, 3>(m, a, n_chunks, s, positions);
    case 256 * 8 + 4: return launch_step_t<256, 4>(m, a, n_chunks, s, positions);
    case 512 * 8 + 1: return launch_step_t<512, 1>(m, a, n_chunks, s, positions);
    case 512 * 8 + 2: return launch_step_t<512, 2>(m, a, n_chunks, s, positions);
    default: break;
  }
  return boa_fail(BOA_ERR_UNSUPPORTED, "no kernel for this d_model / weight format");
}

#ifdef BOA_PHASE_PROFILE
int launch_step_profiled(const boa_model* m, StepArgs& a, int n_chunks, cudaStream_t s) {
  unsigned long long* d = nullptr;
  BOA_CUDA(cudaMalloc(&d, PF_SLOTS * sizeof(unsigned long long)));
  BOA_CUDA(cudaMemsetAsync(d, 0, PF_SLOTS * sizeof(unsigned long long), s));
  a.prof = d;
  int rc = launch_step(m, a, n_chunks, s);
  unsigned long long h[PF_SLOTS] = {0};
  if (rc == BOA_OK) {
    cudaMemcpyAsync(h, d, sizeof(h), cudaMemcpyDeviceToHost, s);
    cudaStreamSynchronize(s);
    static const char* names[20] = {"embed", "ln1", "wait_in", "conv", "wait_xp", "xp_epi", "wait_dt", "scan",
                                    "wait_out", "out_ln2", "wait_ff1", "ff1_epi", "wait_ff2", "ff2_epi", "head0_in",
                                    "wait_h0", "head0_epi", "wait_h2", "head2_epi", "coder"};
    fprintf(stderr, "{\"boa_phase_profile\": {\"mode\": %d, \"steps\": %llu, \"tiles\": %llu", a.mode, h[PF_STEPS],
            h[PF_TILES]);
    for (int i = 0; i < 20; ++i) fprintf(stderr, ", \"%s\": %llu", names[i], h[i]);
    fprintf(stderr, ", \"mma_wait_full\": %llu, \"mma_wait_act\": %llu, \"mma_total\": %llu, \"prod_wait_empty\": %llu}}\n",
            h[PF_MMA_WAIT_FULL], h[PF_MMA_WAIT_ACT], h[PF_MMA_TOTAL], h[PF_PROD_WAIT_EMPTY]);
  }
  cudaFree(d);
  a.prof = nullptr;
  return rc;
}
#endif

int workspace_split(const boa_model* m, int n, void* ws, size_t ws_bytes, float4** conv, float4** ssm) {
  const size_t need = boa_model_workspace_bytes(m, n);
  if (!ws || ws_bytes < need) return boa_fail(BOA_ERR_ARG, "workspace too small (see boa_model_workspace_bytes)");
  if (reinterpret_cast<uintptr_t>(ws) % 16) return boa_fail(BOA_ERR_ARG, "workspace must be 16-byte aligned");
  *ssm = reinterpret_cast<float4*>(ws);
  *conv = reinterpret_cast<float4*>(reinterpret_cast<uint8_t*>(ws) + ssm_state_bytes(m, n));
  return BOA_OK;
}

int check_precision(const boa_model* m, int precision, const char* who) {
  if (precision < 11 || precision > 24 || 2 * m->V > (1 << precision))
    return boa_fail(BOA_ERR_ARG, std::string(who) + ": precision out of range");
  return BOA_OK;
}

int check_range(int pos_begin, int pos_end, const char* who) {
  if (pos_begin < 1 || pos_end <= pos_begin)
    return boa_fail(BOA_ERR_ARG, std::string(who) + ": need 1 <= pos_begin < pos_end");
  return BOA_OK;
}

template <int KIND>
static cudaError_t diag_launch(const uint8_t* d_t, const float* d_x, float* d_o, int M, int K, uint32_t* d_e) {
  const int smem = kTileBytes + kCT * tc::OpKind<KIND>::kHiLo * 1024 * tc::OpKind<KIND>::kElemBytes + 64 + 1024;
  cudaError_t e = cudaFuncSetAttribute(k_diag_gemm<KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  k_diag_gemm<KIND><<<1, 256, smem>>>(d_t, d_x, d_o, M, K, d_e);
  return cudaGetLastError();
}

}  // namespace

extern "C" {

BOA_API int boa_model_create(boa_model** out, int d_model, int n_layers, int vocab, const float* host_flat_weights,
                             size_t n_floats, int weight_format, int device) {
  if (!out) return boa_fail(BOA_ERR_ARG, "boa_model_create: null out");
  *out = nullptr;
  if (d_model != 64 && d_model != 256 && d_model != 512)
    return boa_fail(BOA_ERR_UNSUPPORTED, "boa_model_create: d_model must be 64, 256 or 512");
  if (n_layers < 1 || n_layers > 64) return boa_fail(BOA_ERR_ARG, "boa_model_create: n_layers must be in [1, 64]");
  if (vocab < 2 || vocab > 256) return boa_fail(BOA_ERR_ARG, "boa_model_create: vocab must be in [2, 256]");
  if (weight_format < 0 || weight_format > 4) return boa_fail(BOA_ERR_ARG, "boa_model_create: unknown weight format");
  if (!host_flat_weights) return boa_fail(BOA_ERR_ARG, "boa_model_create: null weights");
  if (d_model == 512 && (weight_format == BOA_WEIGHTS_TF32 || weight_format == BOA_WEIGHTS_TF32X3 ||
                         weight_format == BOA_WEIGHTS_F16X2))
    return boa_fail(BOA_ERR_UNSUPPORTED, "boa_model_create: d_model 512 needs 16-bit weights (bf16 or fp16)");
  if (weight_format == BOA_WEIGHTS_F16X2)
    for (size_t i = 0; i < n_floats; ++i)
      if (!(std::fabs(host_flat_weights[i]) < 65504.0f))
        return boa_fail(BOA_ERR_RANGE, "boa_model_create: a weight outside the 2xFP16 range (|w| < 65504); "
                                       "use BOA_WEIGHTS_TF32X3");
  BOA_CUDA(cudaSetDevice(device));
  boa_model* m = new boa_model();
  m->D = d_model; m->L = n_layers; m->V = vocab; m->kind = weight_format; m->device = device;
  m->plan = make_plan(d_model, n_layers, weight_format, 1);
  m->has_split2 = (d_model == 256 && (weight_format == BOA_WEIGHTS_BF16 || weight_format == BOA_WEIGHTS_F16));
  if (m->has_split2) m->plan2 = make_plan(d_model, n_layers, weight_format, 2);
  cudaDeviceGetAttribute(&m->n_sms, cudaDevAttrMultiProcessorCount, device);
  std::vector<uint8_t> tiles, tiles2;
  std::vector<float> params;
  int rc = BOA_ERR_UNSUPPORTED;
  if (d_model == 64) rc = build_model<64>(m, host_flat_weights, n_floats, tiles, tiles2, params);
  if (d_model == 256) rc = build_model<256>(m, host_flat_weights, n_floats, tiles, tiles2, params);
  if (d_model == 512) rc = build_model<512>(m, host_flat_weights, n_floats, tiles, tiles2, params);
  if (rc != BOA_OK) { delete m; return rc; }
  m->params_floats = params.size();
  cudaError_t e = cudaMalloc(&m->d_tiles, tiles.size());
  if (e == cudaSuccess) e = cudaMalloc(&m->d_params, params.size() * 4);
  if (e == cudaSuccess) e = cudaMalloc(&m->d_err, 4);
  if (e == cudaSuccess) e = cudaMemcpy(m->d_tiles, tiles.data(), tiles.size(), cudaMemcpyHostToDevice);
  if (e == cudaSuccess && m->has_split2) {
    e = cudaMalloc(&m->d_tiles2, tiles2.size());
    if (e == cudaSuccess) e = cudaMemcpy(m->d_tiles2, tiles2.data(), tiles2.size(), cudaMemcpyHostToDevice);
  }
  if (e == cudaSuccess) e = cudaMemcpy(m->d_params, params.data(), params.size() * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemset(m->d_err, 0, 4);
  if (e != cudaSuccess) {
    boa_model_destroy(m);
    return boa_fail(BOA_ERR_CUDA, std::string("boa_model_create: ") + cudaGetErrorString(e));
  }
  *out = m;
  return BOA_OK;
}

BOA_API int boa_model_destroy(boa_model* m) {
  if (!m) return BOA_OK;
  cudaSetDevice(m->device);
  cudaFree(m->d_tiles); cudaFree(m->d_tiles2); cudaFree(m->d_params); cudaFree(m->d_err);
  delete m;
  return BOA_OK;
}

BOA_API size_t boa_model_workspace_bytes(const boa_model* m, int n_chunks) {
  if (!m || n_chunks < 1) return 0;
  // state is addressed per CTA tile of up to 32 chunks, so round the count up
  const int n = cdiv(n_chunks, 32) * 32;
  return conv_state_bytes(m, n) + ssm_state_bytes(m, n);
}

BOA_API int boa_model_set_time_block(boa_model* m, int positions) {
  if (!m || (positions != 0 && positions != 1 && positions != 4 && positions != 8))
    return boa_fail(BOA_ERR_ARG, "boa_model_set_time_block: positions must be 0, 1, 4 or 8");
  m->time_block = positions;
  return BOA_OK;
}

BOA_API int boa_model_time_block(const boa_model* m, int n_chunks, int positions, int* positions_per_step) {
  if (!m || n_chunks < 1 || positions < 1 || !positions_per_step)
    return boa_fail(BOA_ERR_ARG, "boa_model_time_block: bad arguments");
  int tb = 0;
  switch (m->D * 8 + m->kind) {
    case 64 * 8 + 0: tb = boa::encode_time_block_t<64, 0>(m, n_chunks, positions); break;
    case 64 * 8 + 1: tb = boa::encode_time_block_t<64, 1>(m, n_chunks, positions); break;
    case 64 * 8 + 2: tb = boa::encode_time_block_t<64, 2>(m, n_chunks, positions); break;
    case 64 * 8 + 3: tb = boa::encode_time_block_t<64, 3>(m, n_chunks, positions); break;
    case 64 * 8 + 4: tb = boa::encode_time_block_t<64, 4>(m, n_chunks, positions); break;
    case 256 * 8 + 0: tb = boa::encode_time_block_t<256, 0>(m, n_chunks, positions); break;
    case 256 * 8 + 1: tb = boa::encode_time_block_t<256, 1>(m, n_chunks, positions); break;
    case 256 * 8 + 2: tb = boa::encode_time_block_t<256, 2>(m, n_chunks, positions); break;
    case 256 * 8 + 3: tb = boa::encode_time_block_t<256, 3>(m, n_chunks, positions); break;
    case 256 * 8 + 4: tb = boa::encode_time_block_t<256, 4>(m, n_chunks, positions); break;
    case 512 * 8 + 1: tb = boa::encode_time_block_t<512, 1>(m, n_chunks, positions); break;
    case 512 * 8 + 2: tb = boa::encode_time_block_t<512, 2>(m, n_chunks, positions); break;
    default: return boa_fail(BOA_ERR_UNSUPPORTED, "no kernel for this d_model / weight format");
  }
  *positions_per_step = tb;
  return BOA_OK;
}

BOA_API int boa_model_info(const boa_model* m, int* d_model, int* n_layers, int* vocab, int* weight_format,
                           size_t* tile_bytes_per_step) {
  if (!m) return boa_fail(BOA_ERR_ARG, "boa_model_info: null handle");
  if (d_model) *d_model = m->D;
  if (n_layers) *n_layers = m->L;
  if (vocab) *vocab = m->V;
  if (weight_format) *weight_format = m->kind;
  if (tile_bytes_per_step) *tile_bytes_per_step = (size_t)m->plan.per_step * kTileBytes;
  return BOA_OK;
}

BOA_API int boa_model_status(boa_model* m, void* stream) {
  if (!m) return boa_fail(BOA_ERR_ARG, "boa_model_status: null handle");
  BOA_CUDA(cudaSetDevice(m->device));
  cudaStream_t s = (cudaStream_t)stream;
  uint32_t e = 0;
  BOA_CUDA(cudaMemcpyAsync(&e, m->d_err, 4, cudaMemcpyDeviceToHost, s));
  BOA_CUDA(cudaStreamSynchronize(s));
  if (e) {
    BOA_CUDA(cudaMemsetAsync(m->d_err, 0, 4, s));
    BOA_CUDA(cudaStreamSynchronize(s));
    if (e & RC_ERR_TIMEOUT) return boa_fail(BOA_ERR_TIMEOUT, "model kernel: a bounded device wait timed out");
    if (e & RC_ERR_OVERFLOW) return boa_fail(BOA_ERR_OVERFLOW, "codec: a compressed stream exceeded its pitch");
    if (e & RC_ERR_SYMBOL) return boa_fail(BOA_ERR_ARG, "codec: symbol outside the vocabulary");
    if (e & RC_ERR_RANGE)
      return boa_fail(BOA_ERR_RANGE, "model kernel: an activation outside the 2xFP16 range (|v| < 65504); the "
                                     "call's outputs are not valid, use BOA_WEIGHTS_TF32X3");
    return boa_fail(BOA_ERR_CUDA, "model kernel: unknown device error bits");
  }
  return BOA_OK;
}

BOA_API int boa_model_logits(boa_model* m, int n, int n_steps, const int32_t* d_tokens, float* d_logits,
                             void* d_workspace, size_t workspace_bytes, void* stream) {
  if (!m || !d_tokens || !d_logits || n < 1 || n_steps < 1) return boa_fail(BOA_ERR_ARG, "boa_model_logits: bad argument");
  BOA_CUDA(cudaSetDevice(m->device));
  StepArgs a{};
  int rc = workspace_split(m, n, d_workspace, workspace_bytes, &a.conv_state, &a.ssm_state);
  if (rc) return rc;
  a.mode = MODE_LOGITS; a.n_chunks = n; a.n_steps = n_steps; a.fresh = 1; a.precision = 16;
  a.tokens = d_tokens; a.logits = d_logits;
  return launch_step(m, a, n, (cudaStream_t)stream);
}

BOA_API int boa_model_step(boa_model* m, int n, const int32_t* d_tokens, float* d_logits, void* d_workspace,
                           size_t workspace_bytes, void* stream) {
  if (!m || !d_tokens || !d_logits || n < 1) return boa_fail(BOA_ERR_ARG, "boa_model_step: bad argument");
  BOA_CUDA(cudaSetDevice(m->device));
  StepArgs a{};
  int rc = workspace_split(m, n, d_workspace, workspace_bytes, &a.conv_state, &a.ssm_state);
  if (rc) return rc;
  a.mode = MODE_LOGITS; a.n_chunks = n; a.n_steps = 1; a.fresh = 0; a.precision = 16;
  a.tokens = d_tokens; a.logits = d_logits;
  return launch_step(m, a, n, (cudaStream_t)stream);
}

BOA_API int boa_codec_encode_range(boa_model* m, int n_chunks, const uint8_t* d_bytes, int64_t in_pitch,
                                   const int32_t* d_lens, int pos_begin, int pos_end, uint32_t* d_words,
                                   int pitch_words, int32_t* d_sizes, int precision, void* d_workspace,
                                   size_t workspace_bytes, void* stream) {
  if (!m || !d_bytes || !d_lens || !d_words || !d_sizes || n_chunks < 1 || pitch_words < 1)
    return boa_fail(BOA_ERR_ARG, "boa_codec_encode: bad argument");
  int rc = check_precision(m, precision, "boa_codec_encode");
  if (rc) return rc;
  if ((rc = check_range(pos_begin, pos_end, "boa_codec_encode_range"))) return rc;
  BOA_CUDA(cudaSetDevice(m->device));
  StepArgs a{};
  rc = workspace_split(m, n_chunks, d_workspace, workspace_bytes, &a.conv_state, &a.ssm_state);
  if (rc) return rc;
  a.mode = MODE_ENCODE; a.n_chunks = n_chunks; a.fresh = pos_begin == 1; a.precision = precision;
  a.pos0 = pos_begin; a.pos1 = pos_end;
  a.bytes = d_bytes; a.in_pitch = in_pitch; a.lens = d_lens;
  a.words = d_words; a.pitch_words = pitch_words; a.sizes = d_sizes;
  return launch_step(m, a, n_chunks, (cudaStream_t)stream);
}

BOA_API int boa_codec_encode(boa_model* m, int n_chunks, const uint8_t* d_bytes, int64_t in_pitch,
                             const int32_t* d_lens, uint32_t* d_words, int pitch_words, int32_t* d_sizes,
                             int precision, void* d_workspace, size_t workspace_bytes, void* stream) {
  return boa_codec_encode_range(m, n_chunks, d_bytes, in_pitch, d_lens, 1, INT_MAX, d_words, pitch_words, d_sizes,
                                precision, d_workspace, workspace_bytes, stream);
}

BOA_API int boa_codec_decode_range(boa_model* m, int n_chunks, const uint32_t* d_words, int pitch_words,
                                   const int32_t* d_sizes, const int32_t* d_lens, int pos_begin, int pos_end,
                                   const uint8_t* d_prev_bytes, uint8_t* d_out, int64_t out_pitch, int precision,
                                   void* d_workspace, size_t workspace_bytes, void* stream) {
  if (!m || !d_words || !d_sizes || !d_lens || !d_prev_bytes || !d_out || n_chunks < 1 || pitch_words < 1)
    return boa_fail(BOA_ERR_ARG, "boa_codec_decode: bad argument");
  int rc = check_precision(m, precision, "boa_codec_decode");
  if (rc) return rc;
  if ((rc = check_range(pos_begin, pos_end, "boa_codec_decode_range"))) return rc;
  BOA_CUDA(cudaSetDevice(m->device));
  StepArgs a{};
  rc = workspace_split(m, n_chunks, d_workspace, workspace_bytes, &a.conv_state, &a.ssm_state);
  if (rc) return rc;
  a.mode = MODE_DECODE; a.n_chunks = n_chunks; a.fresh = pos_begin == 1; a.precision = precision;
  a.pos0 = pos_begin; a.pos1 = pos_end;
  a.words_in = d_words; a.pitch_words = pitch_words; a.sizes_in = d_sizes; a.lens = d_lens;
  a.first_bytes = d_prev_bytes; a.out = d_out; a.out_pitch = out_pitch;
  return launch_step(m, a, n_chunks, (cudaStream_t)stream);
}

BOA_API int boa_codec_decode(boa_model* m, int n_chunks, const uint32_t* d_words, int pitch_words,
                             const int32_t* d_sizes, const int32_t* d_lens, const uint8_t* d_first_bytes,
                             uint8_t* d_out, int64_t out_pitch, int precision, void* d_workspace,
                             size_t workspace_bytes, void* stream) {
  return boa_codec_decode_range(m, n_chunks, d_words, pitch_words, d_sizes, d_lens, 1, INT_MAX, d_first_bytes, d_out,
                                out_pitch, precision, d_workspace, workspace_bytes, stream);
}

// Every wait in the kernels is bounded: when the budget runs out the waiting
// thread raises the abort flag, the kernel winds down and the host reports
// BOA_ERR_TIMEOUT with the context still usable.  This entry point exercises
// that path on purpose: one thread waits on an mbarrier nothing arrives at.
__global__ void k_diag_timeout(long long budget, uint32_t* err) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    abort_flag = 0;
    tc::fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !tc::mbar_wait(&bar, 0, &abort_flag, budget)) atomicOr(err, RC_ERR_TIMEOUT);
  __syncthreads();
}

BOA_API int boa_diag_timeout(int64_t budget_cycles, int device) {
  if (budget_cycles < 1000 || budget_cycles > 20000000000LL)
    return boa_fail(BOA_ERR_ARG, "boa_diag_timeout: budget out of range");
  BOA_CUDA(cudaSetDevice(device));
  uint32_t* d_e = nullptr;
  cudaError_t e = cudaMalloc(&d_e, 4);
  if (e == cudaSuccess) e = cudaMemset(d_e, 0, 4);
  if (e == cudaSuccess) {
    k_diag_timeout<<<1, 64>>>((long long)budget_cycles, d_e);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  uint32_t err = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&err, d_e, 4, cudaMemcpyDeviceToHost);
  cudaFree(d_e);
  if (e != cudaSuccess) return boa_fail(BOA_ERR_CUDA, std::string("boa_diag_timeout: ") + cudaGetErrorString(e));
  if (err & RC_ERR_TIMEOUT) return boa_fail(BOA_ERR_TIMEOUT, "boa_diag_timeout: the bounded wait ran out");
  return BOA_OK;
}

BOA_API int boa_diag_gemm(int weight_format, int M, int K, const float* h_w, const float* h_x, float* h_out,
                          int device) {
  if (weight_format < 0 || weight_format > 4) return boa_fail(BOA_ERR_ARG, "boa_diag_gemm: bad format");
  const int per = (weight_format == 0 || weight_format == 3) ? 32 : 64;
  if (M < 128 || M % 128 || K < per || K % per || K > 1024 || M > 512)
    return boa_fail(BOA_ERR_ARG, "boa_diag_gemm: M in {128..512} step 128, K multiple of the slice, <= 1024");
  BOA_CUDA(cudaSetDevice(device));
  std::vector<uint8_t> tiles;
  {
    std::vector<MTile> v;
    add_mtiles(v, h_w, M, K, K, 0, M / 128);
    pack_gemm(tiles, v, K / per, weight_format, false);   // M tile by M tile, as k_diag_gemm reads them
  }
  uint8_t* d_t = nullptr; float *d_x = nullptr, *d_o = nullptr; uint32_t* d_e = nullptr;
  cudaError_t e = cudaMalloc(&d_t, tiles.size());
  if (e == cudaSuccess) e = cudaMalloc(&d_x, (size_t)kCT * K * 4);
  if (e == cudaSuccess) e = cudaMalloc(&d_o, (size_t)M * kCT * 4);
  if (e == cudaSuccess) e = cudaMalloc(&d_e, 4);
  if (e == cudaSuccess) e = cudaMemcpy(d_t, tiles.data(), tiles.size(), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(d_x, h_x, (size_t)kCT * K * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemset(d_e, 0, 4);
  if (e == cudaSuccess) {
    if (weight_format == 0) e = diag_launch<0>(d_t, d_x, d_o, M, K, d_e);
    else if (weight_format == 1) e = diag_launch<1>(d_t, d_x, d_o, M, K, d_e);
    else if (weight_format == 2) e = diag_launch<2>(d_t, d_x, d_o, M, K, d_e);
    else if (weight_format == 3) e = diag_launch<3>(d_t, d_x, d_o, M, K, d_e);
    else e = diag_launch<4>(d_t, d_x, d_o, M, K, d_e);
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  uint32_t err = 0;
  if (e == cudaSuccess) e = cudaMemcpy(h_out, d_o, (size_t)M * kCT * 4, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) e = cudaMemcpy(&err, d_e, 4, cudaMemcpyDeviceToHost);
  cudaFree(d_t); cudaFree(d_x); cudaFree(d_o); cudaFree(d_e);
  if (e != cudaSuccess) return boa_fail(BOA_ERR_CUDA, std::string("boa_diag_gemm: ") + cudaGetErrorString(e));
  if (err) return boa_fail(BOA_ERR_TIMEOUT, "boa_diag_gemm: bounded wait timed out");
  return BOA_OK;
}

}  // extern "C"
