// BoaConstrictor model + fused codec loop for sm_100a: the kernel template and
// its launch helpers.  The explicit instantiations live in model_inst_*.cu (one
// translation unit per operand kind, so they compile in parallel); model.cu
// holds the host side and the C-ABI.
//
// What it computes, per byte and per chunk (paths relative to the reference
// project root):
//   h = Emb[prev]                                             model.py:111
//   per block (model.py:57-65):  u = LN1(h)
//     Mamba step (mamba_ssm.Mamba.step; op order also in
//     portability_solved_cpp/boa_gpu.hpp:188-218, mamba_kernels.cu:158-192,264-338):
//       [x,z] = u W_in^T ; conv shift + SiLU -> xc ; [dtr,B,C] = xc W_x^T ;
//       dt = softplus(dtr W_dt^T + b_dt) ; h_n = exp(dt A_n) h_n + dt B_n xc ;
//       y = C.h + D xc ; y *= SiLU(z) ; o = y W_out^T
//     v = LN2(o) ; h += W2 GELU(W1 v + b1) + b2                 model.py:52-56
//   logits = W_h2 ReLU(W_h1 h + b_h1) + b_h2                    model.py:90-95
//   then quantiser + range coder (codec.py:63-76 / 131-141).
//
// Design (B200-first, not a port): one persistent CTA (or a 2-CTA cluster
// splitting the output features) owns CT operand columns and runs every
// timestep of every layer for them; clusters never talk to each other because
// the whole step is row-local per chunk.  A value column is one chunk, or, in
// the time-blocked encode / logits form, one of TB consecutive positions of
// a chunk (TB = 4 or 8).  With the split operand kinds every
// value column occupies two (3xTF32: tf32 hi and lo) or four (2xFP16: hi, lo',
// hi, zero) operand rows, so a tile of CT operand columns holds CT / 2 or
// CT / 4 value columns.  Roles inside the CTA (five warpgroups):
//   warp 0      streams every projection weight tile (pre-packed 16 KB SW128
//               images, in consumption order) through a shared-memory ring
//               with bulk async copies;
//   warp 1      allocates TMEM and issues tcgen05.mma: weights are the A
//               operand (M = 128 output features per tile), the chunks'
//               activations the B operand (N = CT), accumulators in TMEM;
//   warp 2      (single-CTA kernels) a second issuer: the M tiles of every
//               GEMM alternate between warps 1 and 2;
//   warp 3      idle (completes warpgroup 0);
//   warps 4-19  (512 threads) run the LayerNorms, conv/scan/gate, MLP and head
//               epilogues straight out of TMEM, write the next B operand into
//               shared memory, and run quantiser + range coder (a warp per chunk).
// The recurrent state (conv window + SSM state, fp32) streams from HBM once
// per layer per kernel step (per TB bytes); everything else stays on chip.  Every accumulator column
// depends only on its own chunk and the weights, in a fixed K order, so the
// probabilities do not depend on batch composition, grid size or GPU.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "boa_b200.h"
#include "capi_util.h"
#include "rc_device.cuh"
#include "tc_sm100.cuh"

// Lanes of the producer warp that issue weight-tile copies (see the producer).
// 0 (the default) picks them per kernel; a positive value forces that count.
#ifndef BOA_TILE_PRODUCERS
#define BOA_TILE_PRODUCERS 0
#endif

namespace boa {

constexpr int kTileBytes = 16384;      // one A tile: 128 rows x 128 bytes
// Threads per CTA: five warpgroups.  Warpgroup 0 holds the weight producer
// (warp 0), the MMA issuer (warp 1), in single-CTA kernels a second issuer
// (warp 2), and an idle warp; warpgroups 1-4 are the 16 compute warps.  The
// block launches with kRegsLaunch registers a thread; warpgroup 0 then gives
// all but kRegsCtl of them back (setmaxnreg) and the compute warpgroups take
// them, so the epilogues, the scan and the coder run with kRegsCompute.
constexpr int kComputeThreads = 512;   // warps 4..19
constexpr int kComputeWarps = kComputeThreads / 32;
constexpr int kComputeWarp0 = 4;       // first compute warp
constexpr int kIssuer2Warp = 2;        // second MMA issuer (single-CTA kernels)
__host__ __device__ constexpr int threads_for(int) { return 640; }
constexpr int kRegsLaunch = 96, kRegsCtl = 64, kRegsCompute = 104;
static_assert(kRegsCtl * 128 + kRegsCompute * kComputeThreads == kRegsLaunch * 640,
              "the warpgroups' register shares must add up to the launch's");
constexpr long long kWaitBudget = 4000000000LL;  // SM clock cycles per bounded wait (~2 s)

enum StepMode : int { MODE_ENCODE = 0, MODE_DECODE = 1, MODE_LOGITS = 2 };

// Per-layer small parameters (fp32), packed by the host in this order.
template <int D>
struct LayerParams {
  static constexpr int E = 2 * D, F = 4 * D;
  static constexpr int ln1w = 0, ln1b = D, convw = 2 * D, convb = convw + 4 * E, dtb = convb + E,
                       A2 = dtb + E, Dp = A2 + 16 * E, ln2w = Dp + E, ln2b = ln2w + D, b1 = ln2b + D,
                       b2 = b1 + F, stride = b2 + D;
};

static inline int cdiv(int a, int b) { return (a + b - 1) / b; }

// Projection tile counts per step for one CTA of a `split`-way cluster (must
// match the kernel's consumption order; every rank streams the same count).
// With the split operand kinds (3, 4) every (M tile, K slice) is two tiles: hi, lo.
struct TilePlan {
  int per, kD, kE, kF, mtE, mtD, mtF;
  int split, ltE, ltD, ltF, ltV, hl;
  int per_layer, per_step;
};
static inline TilePlan make_plan(int D, int L, int kind, int split) {
  TilePlan p{};
  p.per = (kind == 0 || kind == 3) ? 32 : 64;
  p.hl = (kind == 3 || kind == 4) ? 2 : 1;
  const int E = 2 * D, F = 4 * D;
  p.kD = D / p.per; p.kE = E / p.per; p.kF = F / p.per;
  p.mtE = E / 128; p.mtD = cdiv(D, 128); p.mtF = F / 128;
  p.split = split;
  p.ltE = p.mtE / split; p.ltD = p.mtD / split; p.ltF = p.mtF / split; p.ltV = 2 / split;
  p.per_layer = p.hl * (2 * p.ltE * p.kD + p.kE + p.ltE + p.ltD * p.kE + p.ltF * p.kD + p.ltD * p.kF);
  p.per_step = p.per_layer * L + p.hl * (p.ltD * p.kD + p.ltV * p.kD);
  return p;
}

struct StepArgs {
  int mode;                 // StepMode
  int n_layers;
  int vocab;
  int n_chunks;
  int n_steps;              // logits mode: tokens per stream
  int fresh;                // 1: first step starts from zero state (no state loads)
  int precision;
  int tiles_per_step;
  int tiles_per_layer;
  // encode / decode: positions [pos0, pos1) of every chunk are coded (pos0 >= 1);
  // byte rows (input or output) hold positions [pos0 - 1, pos1): slot 0 is the
  // byte before the range
  int pos0, pos1;
  // encode input
  const uint8_t* bytes; long long in_pitch;
  const int32_t* lens;
  // decode input / output
  const uint32_t* words_in; const int32_t* sizes_in; const uint8_t* first_bytes;
  uint8_t* out; long long out_pitch;
  // encode output
  uint32_t* words; int pitch_words; int32_t* sizes;
  // logits mode
  const int32_t* tokens; float* logits;
  // model
  const uint8_t* wtiles; const float* params;
  float4* conv_state; float4* ssm_state;
  uint32_t* err;
  unsigned long long* prof;   // optional per-phase SM-cycle totals of CTA 0 (BOA_PHASE_PROFILE)
};

// Phase slots of the optional profile (see boa_b200/_native.py PHASES).
enum ProfSlot : int {
  PF_EMBED = 0, PF_LN1, PF_W_IN, PF_CONV, PF_W_XP, PF_XP, PF_W_DT, PF_SCAN, PF_W_OUT, PF_LN2, PF_W_FF1, PF_FF1,
  PF_W_FF2, PF_FF2, PF_HEAD0, PF_W_H0, PF_HEAD1, PF_W_H2, PF_HEAD2, PF_CODER,
  PF_MMA_WAIT_FULL = 24, PF_MMA_WAIT_ACT, PF_MMA_TOTAL, PF_PROD_WAIT_EMPTY, PF_TILES, PF_STEPS, PF_SLOTS = 32
};

// ------------------------------ device math ---------------------------------
__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float softplus_f(float x) { return x > 20.0f ? x : log1pf(expf(x)); }
__device__ __forceinline__ float gelu_f(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }

__device__ __forceinline__ void cbar_sync() {   // named barrier over the 512 compute threads
  asm volatile("bar.sync 1, 512;" ::: "memory");
}

// Operand columns per CTA (the MMA N) is 16 or 32.  A tcgen05.mma with M = 128
// costs about the same for any N <= 128 (the weight tile read dominates), so
// more columns per CTA amortise the weight stream; 32 fits TMEM and shared
// memory with 16-bit operands and d_model <= 256, and with the split kind
// (whose hi/lo halves double the columns of every value).  The host picks 32
// only when there are enough chunks to keep every SM busy.
template <int D, int KIND>
struct ChunkTileMax {
  static constexpr int value = KIND == 4 ? (D == 64 ? 64 : 32) : (KIND == 3 || (KIND != 0 && D <= 256)) ? 32 : 16;
};

// Shared-memory carve-up (dynamic smem, base rounded up to 1024 bytes).
//   SPLIT == 1: one operand buffer; the fp32 scratch (LN2 input / logits)
//               aliases its upper part when it fits (the operand there has
//               been consumed whenever the scratch is written).
//   SPLIT == 2: two operand buffers used alternately by consecutive GEMMs, so
//               the peer CTA can write the next operand while this CTA's
//               tensor core may still read the current one; separate scratch.
// Operand buffers hold CT rows (operand columns); the fp32 arrays hold VC rows
// (value columns: CT / 2 with the split kind).
template <int D, int KIND, int CT_, int SPLIT>
struct Smem {
  static constexpr int CT = CT_;
  static constexpr int VC = CT / tc::OpKind<KIND>::kHiLo;
  static constexpr int EB = tc::OpKind<KIND>::kElemBytes;
  static constexpr int E = 2 * D, F = 4 * D;
  static constexpr int BBUF = CT * F * EB;                  // largest K is F
  static constexpr int NBUF = SPLIT;
  static constexpr int Y_BYTES = CT * E * EB;               // out_proj input (also covers LN2 / head inputs)
  static constexpr int SCR = VC * (D > 256 ? D : 256) * 4;  // LN2 input / logits (fp32)
  static constexpr bool SCR_ALIAS = SPLIT == 1 && BBUF - Y_BYTES >= SCR;
  static constexpr int HRES = VC * D * 4;
  static constexpr int DBCB = VC * 64 * 4;
  static constexpr int o_bbuf = 0;
  static constexpr int o_scr = SCR_ALIAS ? Y_BYTES : NBUF * BBUF;
  static constexpr int o_hres = SCR_ALIAS ? BBUF : NBUF * BBUF + SCR;
  static constexpr int o_dbc = o_hres + HRES;
  static constexpr int o_enc = o_dbc + DBCB;                 // RcEnc / RcDec [VC]
  static constexpr int o_prev = o_enc + VC * 32;
  static constexpr int o_lens = o_prev + VC * 4;
  static constexpr int o_bars = o_lens + VC * 4;
  static constexpr int kMaxStages = 12;
  static constexpr int kTileBars = 16;                      // per-M-tile completion barriers
  static constexpr int o_misc = o_bars + (2 * kMaxStages + 4 + kTileBars) * 8;
  static constexpr int o_prof = o_misc + 64;                 // PF_SLOTS x u64 phase accumulators
  static constexpr int o_ring = ((o_prof + 256 + 1023) / 1024) * 1024;
  static constexpr int kBudget = 227 * 1024 - 1024;          // minus alignment slack
  // The split kinds take each (M tile, K slice) as a hi tile and a lo tile,
  // consecutive in the weight stream and multiplied by the same issuer: a
  // ring slot then holds the pair (one wait, 8 MMAs, one release), where at
  // least 4 pair slots fit.
  static constexpr bool PAIR = tc::OpKind<KIND>::kHiLo >= 2 && (kBudget - o_ring) / (2 * kTileBytes) >= 4;
  static constexpr int SLOT = (PAIR ? 2 : 1) * kTileBytes;
  static constexpr int STAGES_FIT = (kBudget - o_ring) / SLOT;
  static constexpr int STAGES = STAGES_FIT > kMaxStages ? kMaxStages : STAGES_FIT;
  static constexpr int TOTAL = o_ring + STAGES * SLOT;
  static constexpr int ALLOC = TOTAL + 1024;
  static_assert(STAGES >= 3, "not enough shared memory for the weight ring");
};

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// ----------------------------- cluster helpers ------------------------------
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory byte in CTA `peer` of this cluster.
__device__ __forceinline__ uint32_t peer_addr(const void* local, uint32_t peer) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(tc::smem_u32(local)), "r"(peer));
  return r;
}
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t remote_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote_bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(tc::smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                                  long long budget) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > budget) {
      *abort_flag = 1;
      return false;
    }
  }
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_cluster() {
  asm volatile("fence.proxy.async.shared::cluster;" ::: "memory");
}

// -------------------------------- the kernel --------------------------------
// SPLIT == 2 runs as clusters of two CTAs over the same chunk tile: CTA r
// computes output features / channels [r/2, (r+1)/2) of every projection
// (x_proj, whose output is tiny, runs whole in both), streams only its half of
// the weights, and writes every value the peer needs into the peer's shared
// memory as well (DSMEM).  LayerNorms and the coder run redundantly in both
// CTAs on identical data; CTA 0 writes the codec outputs.
// TB > 1 is the time-blocked form of encode and logits mode: the VC value
// columns are VC / TB chunks x TB consecutive positions (column n = chunk
// n / TB, position offset n % TB), so one pass of the weights serves TB
// positions and each chunk's recurrent state is read and written once per TB
// positions.  The conv window and the SSM state carry from one position to
// the next in registers, and every column goes through the same arithmetic
// as in the one-position step, so the logits, and hence the bitstream, are
// bit for bit those of the TB = 1 kernel that decode uses.
template <int D, int KIND, int CT_, int SPLIT, int TB>
__global__ void __launch_bounds__(threads_for(SPLIT), 1) k_boa_step(const __grid_constant__ StepArgs a) {
  using S = Smem<D, KIND, CT_, SPLIT>;
  using LP = LayerParams<D>;
  constexpr int CT = S::CT;                              // operand columns (the MMA N)
  constexpr int HL = tc::OpKind<KIND>::kHiLo;            // operand columns per value column
  constexpr int VC = S::VC;                              // value columns
  constexpr int CHUNKS = VC / TB;                        // chunks per CTA (per cluster when SPLIT == 2)
  static_assert(TB == 1 || TB == 2 || TB == 4 || TB == 8, "time block");
  static_assert(TB == 1 || SPLIT == 1, "time blocks run on single CTAs");
  static_assert(HL == 1 || SPLIT == 1, "the split operand kinds run on single CTAs");
  static_assert(VC % 8 == 0 && VC <= 32, "value columns");
  constexpr int NG = VC / 8;                             // groups of 8 value columns
  constexpr int kStagesK = S::STAGES;
  // copy lanes of warp 0: one with pair slots (32 KB copies) and in general;
  // two where measured faster with 16 KB slots (2xFP16, 3xTF32 decode)
  constexpr int kProdWant = BOA_TILE_PRODUCERS > 0 ? BOA_TILE_PRODUCERS
                            : S::PAIR                         ? 1
                            : (KIND == 4 || (KIND == 3 && TB == 1)) ? 2
                                                                    : 1;
  constexpr int kProducers = kStagesK < kProdWant ? kStagesK : kProdWant;
  // Issuing a tcgen05.mma costs the issuing thread about as long as the tensor
  // core needs for it at N <= 64, so single-CTA kernels (whose GEMMs have two
  // or more M tiles) issue from two threads.  Each issuer walks the whole tile
  // sequence and issues the M tiles mt with mt % 2 == its index; every
  // accumulator still sums its K slices in the same order.
  constexpr int kIssuers = SPLIT == 1 ? 2 : 1;
  // With two consumers of one ring an issuer skips the other's tiles and may
  // reach a slot a whole ring round ahead of it, where the full barrier's
  // phase parity alone would be ambiguous.  The producer therefore records,
  // per slot, the (16-bit) index of the tile it is loading after the slot's
  // previous tile was consumed; an issuer first waits for its tile's index in
  // the slot, after which the parity wait is exact.
  constexpr int E = 2 * D, R = (D + 15) / 16, DBC = R + 32, F = 4 * D;
  constexpr int PER = 128 / tc::OpKind<KIND>::kElemBytes;
  constexpr int kD = D / PER, kE = E / PER, kF = F / PER;
  constexpr int MT_E = E / 128, MT_D = (D + 127) / 128, MT_F = F / 128;
  // tiles owned by this CTA
  constexpr int LT_E = MT_E / SPLIT, LT_D = MT_D / SPLIT, LT_F = MT_F / SPLIT, LT_V = 2 / SPLIT;
  static_assert(SPLIT == 1 || (MT_E % 2 == 0 && MT_D % 2 == 0), "split needs an even number of tiles");
  // x_proj has one M tile; its K runs as two halves into two accumulators
  // (COL_XP, COL_XP + CT), one per MMA issuer, summed in the epilogue
  constexpr int COL_X = 0, COL_Z = LT_E * CT, COL_XP = 2 * LT_E * CT, COL_DT = COL_XP + 2 * CT;
  static_assert(COL_DT + LT_E * CT <= 512, "TMEM budget");
  static_assert(LT_F * CT <= 512, "TMEM budget (ff.0)");
  static_assert(R <= PER && DBC <= 64, "x_proj outputs must fit one tile / one K slice");
  static_assert(D % 32 == 0 && D >= 64, "d_model");
  // per-channel phases: (tile, chunk run) units spread over the 4 warp groups
  constexpr int RUNS = LT_E >= 4 ? 1 : 4 / LT_E;         // value-column runs per local channel tile
  constexpr int RUN = VC / RUNS;
  static_assert(RUN % 4 == 0 && RUN >= 4, "chunk run");
  static_assert(RUN % TB == 0, "a chunk run holds whole time blocks");
  // Tile pipelining: the conv starts on finished in_proj M tiles, the GELU on
  // finished ff.0 tiles, so the epilogue's writes of the next operand must not
  // touch the operand the remaining tiles still read.  With two buffers the
  // next operand goes to the other one.  With one buffer the x_proj operand
  // (K = E) is placed after in_proj's (K = D) -- (D + E) <= F slices fit the
  // buffer -- and the GELU tiles that would overwrite ff.0's operand wait for
  // the whole GEMM.
  constexpr int kXOff = S::NBUF == 1 ? kD : 0;           // x_proj operand offset, K slices
  // first ff.0 M tile whose GELU output (K slices [t*128/PER, (t+1)*128/PER)
  // of the ff.2 operand) misses ff.0's operand (slices [0, kD)) in one buffer
  constexpr int kSafeTile = S::NBUF == 2 ? 0 : (D + 127) / 128;
  // value-column masks: first / last position of each chunk's time block
  constexpr uint32_t kColAll = VC == 32 ? 0xffffffffu : ((1u << VC) - 1u);
  constexpr uint32_t kFirstCols = [] {
    uint32_t m = 0;
    for (int n = 0; n < VC; n += TB) m |= 1u << n;
    return m;
  }();
  constexpr uint32_t kLastCols = (kFirstCols << (TB - 1)) & kColAll;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem + S::o_ring;
  uint8_t* bbuf0 = smem + S::o_bbuf;
  float* hres = reinterpret_cast<float*>(smem + S::o_hres);
  float* scr = reinterpret_cast<float*>(smem + S::o_scr);
  float* dbc = reinterpret_cast<float*>(smem + S::o_dbc);
  int32_t* prev = reinterpret_cast<int32_t*>(smem + S::o_prev);
  int32_t* lens_sh = reinterpret_cast<int32_t*>(smem + S::o_lens);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::o_bars);
  uint64_t* empty = full + S::kMaxStages;
  uint64_t* mma_bar = empty + S::kMaxStages;
  uint64_t* act_bar = mma_bar + 1;
  uint64_t* drain_bar = act_bar + 1;
  uint64_t* xch_bar = drain_bar + 1;                      // peer finished writing an exchange
  uint64_t* tile_bar = xch_bar + 1;                       // in_proj / ff.0: M tile t done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::o_misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + S::o_misc + 4);
  int* nsteps_sh = reinterpret_cast<int*>(smem + S::o_misc + 8);
  volatile uint16_t* slot_tile = reinterpret_cast<volatile uint16_t*>(smem + S::o_misc + 24);   // [kMaxStages]
  // per ring slot: phase parity of the newest copy issued into it (0xff: none)
  volatile uint8_t* slot_ph = reinterpret_cast<volatile uint8_t*>(smem + S::o_misc + 48);      // [kMaxStages]

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const uint32_t rank = SPLIT == 2 ? cluster_rank() : 0u;
  const uint32_t peer = rank ^ 1u;
  const int c0 = (blockIdx.x / SPLIT) * CHUNKS;         // first chunk; value column n codes chunk c0 + n / TB
  const int mode = a.mode;
  const int L = a.n_layers;
  const int V = a.vocab;
  const float* P = a.params;
  const long long o_bh0 = (long long)LP::stride * L;
  const long long o_bh2 = o_bh0 + D;
  const long long o_emb = o_bh2 + 256;
  const bool writer = rank == 0;                          // writes the codec outputs
  // encode / decode: the first coded position and the position that byte row
  // slot 0 holds (byte rows cover positions [pos0 - 1, pos1))
  const int pos0 = mode == MODE_LOGITS ? 0 : a.pos0;
  const int origin = mode == MODE_LOGITS ? 0 : a.pos0 - 1;

  // ------------------------------- setup -------------------------------
  if (tid == 0) {
    for (int s = 0; s < kStagesK; ++s) { tc::mbar_init(&full[s], 1); tc::mbar_init(&empty[s], 1); }
    tc::mbar_init(mma_bar, kIssuers);                     // each issuer commits once per GEMM
    tc::mbar_init(act_bar, kComputeWarps * SPLIT);        // both CTAs' compute warps (lane 0 of each)
    tc::mbar_init(drain_bar, kIssuers);
    tc::mbar_init(xch_bar, kComputeWarps);                // the peer's compute warps
    for (int t = 0; t < S::kTileBars; ++t) tc::mbar_init(&tile_bar[t], 1);
    *abort_flag = 0;
    for (int s = 0; s < S::kMaxStages; ++s) slot_ph[s] = 0xffu;
    if constexpr (kIssuers == 2)
      for (int s = 0; s < S::kMaxStages; ++s) slot_tile[s] = 0xffffu;
    int ns = 0;
    if (mode == MODE_LOGITS) {
      ns = a.n_steps;
    } else {
      for (int n = 0; n < CHUNKS; ++n) {
        const int c = c0 + n;
        if (c < a.n_chunks) ns = max(ns, min(a.lens[c], a.pos1) - pos0);
      }
    }
    *nsteps_sh = (ns + TB - 1) / TB;                      // steps of TB positions
    tc::fence_barrier_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  if (tid >= 64 && tid < 64 + VC) {
    const int n = tid - 64;
    const int c = c0 + n / TB, jj = n % TB;
    int p0 = 0, len = 0;
    if (c < a.n_chunks) {
      if (mode == MODE_ENCODE) {
        len = min(a.lens[c], a.pos1);                     // end of this launch's range
        const int t = pos0 - 1 + jj;                      // input of column jj's first position
        p0 = t < len ? a.bytes[(long long)c * a.in_pitch + (t - origin)] : 0;
        if (jj == 0) rc_enc_reset(reinterpret_cast<RcEnc*>(smem + S::o_enc)[n / TB]);
      } else if (mode == MODE_DECODE) {
        len = min(a.lens[c], a.pos1);
        p0 = a.first_bytes[c];                            // the byte at pos0 - 1
        int nw = a.sizes_in[c];
        nw = nw < 0 ? 0 : (nw > a.pitch_words ? a.pitch_words : nw);
        rc_dec_reset(reinterpret_cast<RcDec*>(smem + S::o_enc)[n], a.words_in + (long long)c * a.pitch_words, nw);
        if (writer && pos0 - 1 < a.lens[c]) a.out[(long long)c * a.out_pitch] = (uint8_t)p0;
      } else {
        len = a.n_steps;
        p0 = jj < a.n_steps ? a.tokens[(long long)c * a.n_steps + jj] : 0;
      }
    }
    prev[n] = (p0 >= 0 && p0 < V) ? p0 : 0;
    lens_sh[n] = len;     // 0 marks a padding column (no chunk)
  }
  tc::tc_fence_before();
  __syncthreads();
  if constexpr (SPLIT == 2) cluster_sync_all();           // peer barriers initialised before any remote arrive
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nsteps = *nsteps_sh;

  if (warp < kComputeWarp0) {
  tc::setmaxnreg_dec<kRegsCtl>();                         // every warp of warpgroup 0
  if (warp == 0) {
    // ============================== producer ==============================
    // A bulk copy issued by one thread takes about 470 SM cycles whatever its
    // size up to 64 KB, and a thread's copies do not overlap, so one lane
    // streaming 16 KB tiles delivers ~35 B/clk on its own.  kProducers lanes
    // each own the ring slots st with st % kProducers == lane and fill them in
    // slot order, so the copies of different lanes overlap.  Measured at
    // d_model 256 / 8 layers and 1000 chunks: two lanes shorten 2xFP16 encode
    // and decode steps by about 5 % and 3xTF32 decode steps by 9 %, but
    // lengthen 3xTF32 encode steps by 13 % and leave fp16 unchanged; three
    // lanes are slower than two.  Pair slots (S::PAIR, one 32 KB copy of a hi
    // and a lo tile) shortened 2xFP16 encode steps by a further 13 % and
    // decode steps by 6 %: they halve the issuers' waits and releases.  With
    // pair slots one lane is faster again than two (2xFP16: encode 4 %,
    // decode 6 %), so pair-slot kernels take one.
    if (lane < kProducers && nsteps > 0) {
      const uint64_t pol = tc::policy_evict_last();
      bool ok = true;
#ifdef BOA_PHASE_PROFILE
      const bool prof = a.prof != nullptr && blockIdx.x == 0 && lane == 0;
#else
      constexpr bool prof = false;
#endif
      unsigned long long w_empty = 0;
      const uint8_t* base = a.wtiles + (long long)rank * a.tiles_per_step * kTileBytes;
      const int slots_per_step = a.tiles_per_step / (S::PAIR ? 2 : 1);
      const long long total = (long long)nsteps * slots_per_step;
      for (long long r = 0; ok; ++r) {                     // ring rounds
        for (int st = lane; st < kStagesK; st += kProducers) {
          const long long g = r * kStagesK + st;           // slot-load index in consumption order
          if (g >= total) { ok = false; break; }
          const long long tw = prof ? clock64() : 0;
          if (!tc::mbar_wait(&empty[st], (uint32_t)(r & 1) ^ 1u, abort_flag, kWaitBudget)) { ok = false; break; }
          if (prof) w_empty += clock64() - tw;
          if constexpr (kIssuers == 2) slot_tile[st] = (uint16_t)g;
          slot_ph[st] = (uint8_t)(r & 1);
          tc::mbar_arrive_expect_tx(&full[st], S::SLOT);
          tc::bulk_g2s(ring + st * S::SLOT, base + (g % slots_per_step) * S::SLOT, S::SLOT, &full[st], pol);
        }
      }
      if (prof) a.prof[PF_PROD_WAIT_EMPTY] = w_empty;
    }
  } else if (warp == 1 || (kIssuers == 2 && warp == kIssuer2Warp)) {
    // ============================= MMA issuers ============================
    const int p = warp == 1 ? 0 : 1;
    if (lane == 0 && nsteps > 0) {
      // kind 4 multiplies each weight tile by half of the operand rows (§ OpKind<4>)
      const uint32_t id = tc::idesc<KIND>(128, HL == 4 ? CT / 2 : CT);
      const uint64_t adesc0 = tc::sdesc_sw128(tc::smem_u32(ring));
      constexpr uint64_t kTileDesc = kTileBytes >> 4;      // descriptor start-address units (16 B)
      constexpr uint64_t kSlotDesc = S::SLOT >> 4;
      constexpr uint64_t kSliceDesc = (CT * 128) >> 4;
      constexpr uint64_t kBufDesc = S::BBUF >> 4;
      const uint64_t bdesc_base = tc::sdesc_sw128(tc::smem_u32(bbuf0));
      long long it = 0;
      int st = 0;
      uint32_t ph = 0;
      uint32_t act_phase = 0;
      int gemm_no = 0;                                     // selects the operand buffer
      bool ok = true;
#ifdef BOA_PHASE_PROFILE
      const bool prof = a.prof != nullptr && blockIdx.x == 0 && p == 0;
#else
      constexpr bool prof = false;
#endif
      unsigned long long w_full = 0, w_act = 0;
      const long long t_mma0 = clock64();
      // One ring slot: wait for it, issue the four K8 / K16 MMAs of its tile
      // (with pair slots, then the four of its lo tile into dcol2 with bd2),
      // release the slot.
      auto tile_mma = [&](uint32_t dcol, uint64_t bd, bool acc, uint32_t dcol2 = 0, uint64_t bd2 = 0) -> bool {
        const long long tw = prof ? clock64() : 0;
        if constexpr (kIssuers == 2) {                     // the producer has moved this slot on to tile `it`
          const long long t0 = clock64();
          while (slot_tile[st] != (uint16_t)it) {
            if (*abort_flag) return false;
            if (clock64() - t0 > kWaitBudget) { *abort_flag = 1; return false; }
          }
        }
        if (!tc::mbar_wait(&full[st], ph, abort_flag, kWaitBudget)) return false;
        if (prof) w_full += clock64() - tw;
        tc::tc_fence_after();
        const uint64_t ad = adesc0 + (uint64_t)st * kSlotDesc;
        tc::mma<KIND>(dcol, ad, bd, id, acc ? 1u : 0u);
        tc::mma<KIND>(dcol, ad + 2, bd + 2, id, 1u);       // +32 bytes of K
        tc::mma<KIND>(dcol, ad + 4, bd + 4, id, 1u);
        tc::mma<KIND>(dcol, ad + 6, bd + 6, id, 1u);
        if constexpr (S::PAIR) {                           // the lo tile, 16 KB further on
          const uint64_t al = ad + kTileDesc;
          tc::mma<KIND>(dcol2, al, bd2, id, 1u);
          tc::mma<KIND>(dcol2, al + 2, bd2 + 2, id, 1u);
          tc::mma<KIND>(dcol2, al + 4, bd2 + 4, id, 1u);
          tc::mma<KIND>(dcol2, al + 6, bd2 + 6, id, 1u);
        }
        tc::mma_commit(&empty[st]);
        return true;
      };
      auto next_tile = [&]() {
        ++it;
        if (++st == kStagesK) { st = 0; ph ^= 1u; }
      };
      // D[col0 + mt*CT ...] = sum over ks of A(mt, ks) * B(ks)^T, K slices in order.
      // Cluster kernels take the tiles M tile by M tile; single-CTA kernels
      // take M tiles in pairs with their K slices interleaved (the packing
      // order of their weight stream), tile (2q + h, ks) going to issuer h.
      // With the split kinds each (mt, ks) is the hi tile then the lo tile:
      // kind 3 multiplies both by the whole operand (hi and lo rows), kind 4
      // the hi tile by rows [0, 2 VC) and the lo' tile by rows [2 VC, 4 VC).
      // tiles: also commit after every M tile (pair), so the epilogue of a
      // finished tile can start while later tiles run (in_proj -> conv, ff.0 -> GELU)
      // b_mt: operand K slices between consecutive M tiles (x_proj's two K halves)
      auto gemm = [&](int n_mt, int n_ks, int col0, bool tiles, int b_off, int b_mt) -> bool {
        const uint64_t bdesc0 = bdesc_base + (uint64_t)(gemm_no % S::NBUF) * kBufDesc + (uint64_t)b_off * kSliceDesc;
        constexpr int kGroup = SPLIT == 1 ? 2 : 1;          // M tiles whose K slices interleave
        for (int m0 = 0; m0 < n_mt; m0 += kGroup) {
          const int nm = n_mt - m0 < kGroup ? n_mt - m0 : kGroup;
          uint64_t bd = bdesc0;
          for (int ks = 0; ks < n_ks; ++ks, bd += kSliceDesc) {
            for (int h = 0; h < nm; ++h) {
              const int mt = m0 + h;
              // kind 4: the lo' tile takes operand rows [2 VC, 4 VC) into columns [VC, 3 VC)
              const uint32_t dc_hi = tmem + (uint32_t)(col0 + mt * CT);
              const uint32_t dc_lo = dc_hi + (HL == 4 ? (uint32_t)VC : 0u);
              const uint64_t bd_hi = bd + (uint64_t)(mt * b_mt) * kSliceDesc;
              const uint64_t bd_lo = bd_hi + (HL == 4 ? (uint64_t)((2 * VC * 128) >> 4) : 0ull);
              const bool mine = kIssuers == 1 || (mt & 1) == p;
              if constexpr (S::PAIR) {
                if (mine && !tile_mma(dc_hi, bd_hi, ks > 0, dc_lo, bd_lo)) return false;
                next_tile();
              } else {
#pragma unroll
                for (int hl = 0; hl < (HL == 1 ? 1 : 2); ++hl) {
                  if (mine && !tile_mma(hl ? dc_lo : dc_hi, hl ? bd_lo : bd_hi, ks > 0 || hl > 0)) return false;
                  next_tile();
                }
              }
            }
          }
          if (tiles)
            for (int h = 0; h < nm; ++h)
              if (kIssuers == 1 || ((m0 + h) & 1) == p) tc::mma_commit(&tile_bar[m0 + h]);
        }
        return true;
      };
      auto step_gemm = [&](int n_mt, int n_ks, int col0, bool tiles = false, int b_off = 0, int b_mt = 0) -> bool {
        const long long tw = prof ? clock64() : 0;
        const bool got = SPLIT == 2 ? mbar_wait_cluster(act_bar, act_phase, abort_flag, kWaitBudget)
                                    : tc::mbar_wait(act_bar, act_phase, abort_flag, kWaitBudget);
        if (!got) return false;
        if (prof) w_act += clock64() - tw;
        act_phase ^= 1u;
        tc::tc_fence_after();
        if (!gemm(n_mt, n_ks, col0, tiles, b_off, b_mt)) return false;
        tc::mma_commit(mma_bar);                            // one of the kIssuers arrivals that end the GEMM
        ++gemm_no;
        return true;
      };
      for (int s = 0; s < nsteps && ok; ++s) {
        for (int l = 0; l < L && ok; ++l) {
          ok = step_gemm(2 * LT_E, kD, 0, true)    // in_proj -> x | z (own channels)
               && step_gemm(2, kE / 2, COL_XP, false, kXOff, kE / 2)   // x_proj (whole), two K halves
               && step_gemm(LT_E, 1, COL_DT)       // dt_proj (own channels)
               && step_gemm(LT_D, kE, 0)           // out_proj (own features)
               && step_gemm(LT_F, kD, 0, true)     // ff.0
               && step_gemm(LT_D, kF, 0);          // ff.2
        }
        ok = ok && step_gemm(LT_D, kD, 0)          // head.0
             && step_gemm(LT_V, kD, 0);            // head.2
      }
      if (prof) {
        a.prof[PF_MMA_WAIT_FULL] = w_full;
        a.prof[PF_MMA_WAIT_ACT] = w_act;
        a.prof[PF_MMA_TOTAL] = clock64() - t_mma0;
        a.prof[PF_TILES] = (unsigned long long)it;
        a.prof[PF_STEPS] = (unsigned long long)nsteps;
      }
      // every issued MMA (of both issuers) must retire before TMEM is released
      tc::mma_commit(drain_bar);
      const long long t0 = clock64();
      while (!tc::mbar_try_wait(drain_bar, 0)) {
        if (clock64() - t0 > kWaitBudget) break;
      }
    }
  }
  } else {
    tc::setmaxnreg_inc<kRegsCompute>();                   // every compute warp
    // ============================ compute warps ============================
    const int ct = tid - 32 * kComputeWarp0; // 0..511
    const int cw = ct >> 5;                  // compute warp 0..15
    const int q = warp & 3;                  // TMEM lane quarter this warp may access
    const int g = cw >> 2;                   // group 0..3 (covers all four quarters)
    const int row = 32 * q + lane;           // row inside a 128-row M tile
    const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16);
    uint32_t mma_phase = 0, xch_phase = 0;
    int gemm_no = 0;                         // operand buffer of the next GEMM = gemm_no % NBUF
    RcEnc* encs = reinterpret_cast<RcEnc*>(smem + S::o_enc);
    RcDec* decs = reinterpret_cast<RcDec*>(smem + S::o_enc);
    const uint32_t peer_bbuf = SPLIT == 2 ? peer_addr(bbuf0, peer) : 0u;
    const uint32_t peer_hres = SPLIT == 2 ? peer_addr(hres, peer) : 0u;
    const uint32_t peer_scr = SPLIT == 2 ? peer_addr(scr, peer) : 0u;
    const uint32_t peer_act = SPLIT == 2 ? peer_addr(act_bar, peer) : 0u;
    const uint32_t peer_xch = SPLIT == 2 ? peer_addr(xch_bar, peer) : 0u;
#ifdef BOA_PHASE_PROFILE
    const bool pon = a.prof != nullptr && blockIdx.x == 0 && ct == 0;
    unsigned long long* pacc = reinterpret_cast<unsigned long long*>(smem + S::o_prof);
    if (pon) for (int i = 0; i < 20; ++i) pacc[i] = 0;
    long long tlast = clock64();
    auto mark = [&](int slot) {
      if (pon) { const long long now = clock64(); pacc[slot] += (unsigned long long)(now - tlast); tlast = now; }
    };
#else
    auto mark = [](int) {};
#endif
    // Accumulators of eight (four) value columns starting at TMEM column
    // `col` of this warp's lane quarter: one load, or with the split kinds the
    // sum of the columns col and col + VC (scaled by 2^-11 for kind 4).
    auto ldv8 = [&](uint32_t col, float (&v)[8]) {
      if constexpr (HL == 4) tc::tmem_ld8_sum_s11(tq + col, tq + col + VC, v);
      else if constexpr (HL == 2) tc::tmem_ld8_sum(tq + col, tq + col + VC, v);
      else tc::tmem_ld8(tq + col, v);
    };
    auto ldv4 = [&](uint32_t col, float (&v)[4]) {
      if constexpr (HL == 4) tc::tmem_ld4_sum_s11(tq + col, tq + col + VC, v);
      else if constexpr (HL == 2) tc::tmem_ld4_sum(tq + col, tq + col + VC, v);
      else tc::tmem_ld4(tq + col, v);
    };
    // operand buffer the next GEMM reads
    auto bnext = [&]() -> uint8_t* { return bbuf0 + (gemm_no % S::NBUF) * S::BBUF; };
    // write one operand element of the next GEMM (this CTA's copy); kind 4
    // records values its fp16 halves cannot hold (reported as RC_ERR_RANGE)
    bool range_bad = false;
    uint32_t amask_cur = 0;                  // this step's active value columns
    auto put_b = [&](uint8_t* buf, int n, int k, float v) {
      if constexpr (HL == 4) range_bad |= ((amask_cur >> n) & 1u) && !(fabsf(v) < 65504.0f);
      tc::store_operand<KIND>(buf, n, k, CT, v);
    };
    // SPLIT == 2: after all threads wrote this CTA's share of the next operand
    // (K slices [s0, s0 + ns), contiguous in the buffer), copy it into the
    // peer's buffer, 16 bytes per thread and store
    auto push_slices = [&](uint8_t* buf, int s0, int ns) {
      if constexpr (SPLIT == 2) {
        cbar_sync();
        const uint32_t off0 = (uint32_t)(buf - bbuf0) + (uint32_t)(s0 * CT * 128);
        const int bytes = ns * CT * 128;
        for (int o = ct * 16; o < bytes; o += kComputeThreads * 16)
          st_cluster_v4(peer_bbuf + off0 + (uint32_t)o, *reinterpret_cast<const uint4*>(bbuf0 + off0 + o));
      }
    };
    // SPLIT == 2: copy columns [c, c + nf) of the VC rows of an fp32 [VC][row] array into the peer
    auto push_rows = [&](float* arr, uint32_t peer_arr, int row, int c, int nf) {
      if constexpr (SPLIT == 2) {
        cbar_sync();
        const int per_row = nf / 4;
        for (int i = ct; i < VC * per_row; i += kComputeThreads) {
          const int r = i / per_row;
          const int idx = r * row + c + 4 * (i - r * per_row);
          st_cluster_v4(peer_arr + 4u * (uint32_t)idx, *reinterpret_cast<const uint4*>(arr + idx));
        }
      }
    };
    // Every thread orders its operand writes (and TMEM reads) before the
    // warp barrier; lane 0 then arrives once for the warp, which keeps the
    // barrier traffic at 16 arrivals per CTA instead of 512.
    auto arrive_act = [&]() {
      if constexpr (SPLIT == 2) fence_proxy_async_cluster();
      else tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        tc::mbar_arrive(act_bar);
        if constexpr (SPLIT == 2) mbar_arrive_remote(peer_act);
      }
      ++gemm_no;
    };
    // Wait for the GEMM just issued; the result is uniform over the 512 threads.
    auto wait_mma = [&]() -> bool {
      tc::mbar_wait(mma_bar, mma_phase, abort_flag, kWaitBudget);
      mma_phase ^= 1u;
      cbar_sync();
      tc::tc_fence_after();
      return *abort_flag == 0;
    };
    // Per-M-tile completion of in_proj / ff.0: a unit waits for the tile it
    // reads; gemm_done() then waits (usually without spinning) for the whole
    // GEMM, which keeps every barrier's phase parity in step.
    uint32_t tile_ph = 0;
    static_assert(2 * LT_E <= S::kTileBars && LT_F <= S::kTileBars, "tile barriers");
    auto wait_tile = [&](int mt) {
      tc::mbar_wait(&tile_bar[mt], (tile_ph >> mt) & 1u, abort_flag, kWaitBudget);
      tc::tc_fence_after();
    };
    auto gemm_done = [&](int n_mt) {
      tc::mbar_wait(mma_bar, mma_phase, abort_flag, kWaitBudget);
      mma_phase ^= 1u;
      tile_ph ^= (1u << n_mt) - 1u;
      tc::tc_fence_after();
    };
    // After writing shared values into the peer: tell it, then wait for its
    // values to have arrived here.  Uniform result as wait_mma.
    auto exchange = [&]() -> bool {
      if constexpr (SPLIT == 2) {
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(peer_xch);
        mbar_wait_cluster(xch_bar, xch_phase, abort_flag, kWaitBudget);
        xch_phase ^= 1u;
      }
      cbar_sync();
      return *abort_flag == 0;
    };
    // LayerNorm (eps 1e-5, biased variance, two passes) of VC rows of `src`
    // (fp32 [VC][D]) into the next operand; a warp per value column, whole rows.
    auto layernorm_to_b = [&](const float* src, const float* w, const float* b) {
      constexpr int PLN = D / 32;
      uint8_t* buf = bnext();
      for (int n = cw; n < VC; n += 16) {
        float v[PLN];
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < PLN; ++i) { v[i] = src[n * D + lane + 32 * i]; s += v[i]; }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        const float mean = s * (1.0f / D);
        float var = 0.f;
#pragma unroll
        for (int i = 0; i < PLN; ++i) { const float dl = v[i] - mean; var += dl * dl; }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o);
        const float rstd = rsqrtf(var * (1.0f / D) + 1e-5f);
#pragma unroll
        for (int i = 0; i < PLN; ++i) {
          const int f = lane + 32 * i;
          put_b(buf, n, f, (v[i] - mean) * rstd * __ldg(w + f) + __ldg(b + f));
        }
      }
    };

    bool ok = true;
    for (int s = 0; s < nsteps && ok; ++s) {
      // value column n predicts / codes position t0 + n % TB
      const int t0 = (mode == MODE_LOGITS) ? s * TB : pos0 + s * TB;
      const bool load_state = !(a.fresh && s == 0);
      // active mask of this step (bit n: column n codes a position of its chunk)
      uint32_t amask = 0;
#pragma unroll
      for (int n = 0; n < VC; ++n) amask |= (t0 + n % TB < lens_sh[n] ? 1u : 0u) << n;
      amask_cur = amask;
      // state is read at a chunk's first column and written after its last
      // active one, for chunks that are still running in this step
      const uint32_t lmask = load_state ? (amask & kFirstCols) : 0u;
      const uint32_t smask = amask & (kLastCols | ~(amask >> 1));
      // ---- embedding (both CTAs, whole rows)
      for (int i = ct; i < VC * D; i += kComputeThreads) {
        const int n = i / D, f = i - (i / D) * D;
        hres[i] = __ldg(P + o_emb + (long long)prev[n] * D + f);
      }
      cbar_sync();
      mark(PF_EMBED);
      for (int l = 0; l < L && ok; ++l) {
        const float* lp = P + (long long)LP::stride * l;
        // ---- LN1 -> operand ; in_proj
        layernorm_to_b(hres, lp + LP::ln1w, lp + LP::ln1b);
        arrive_act();
        mark(PF_LN1);
        mark(PF_W_IN);
        // ---- causal conv (width 4) + SiLU, thread per own channel; xc -> both
        //      CTAs' operand (x_proj runs whole) and into TMEM for the scan
        {
          uint8_t* buf = bnext() + kXOff * CT * 128;      // x_proj operand (after in_proj's with one buffer)
          for (int u = g; u < LT_E * NG; u += 4) {
            const int lt = u / NG;
            wait_tile(lt);                                // x tile lt of in_proj
            const int e = (int)(rank * LT_E + lt) * 128 + row;
            const float4 w = __ldg(reinterpret_cast<const float4*>(lp + LP::convw) + e);
            const float cb = __ldg(lp + LP::convb + e);
            float4* cs = a.conv_state + ((long long)c0 * L + l) * E + e;   // chunk stride L*E
            const long long cst = (long long)L * E;
            {
              const int nb = (u % NG) * 8;                  // 8 value columns = 8 / TB whole chunks
              float4 stv[8 / TB];
#pragma unroll
              for (int j = 0; j < 8; j += TB)
                stv[j / TB] = ((lmask >> (nb + j)) & 1u) ? __ldcs(&cs[((nb + j) / TB) * cst]) : make_float4(0.f, 0.f, 0.f, 0.f);
              float xv[8];
              const uint32_t col = (uint32_t)(COL_X + lt * CT + nb);
              ldv8(col, xv);
              float4 win = stv[0];                          // window (x[t-3], x[t-2], x[t-1]) of column nb
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const int n = nb + j;
                if (j % TB == 0) win = stv[j / TB];
                float acc = cb;
                acc = fmaf(w.x, win.x, acc);
                acc = fmaf(w.y, win.y, acc);
                acc = fmaf(w.z, win.z, acc);
                acc = fmaf(w.w, xv[j], acc);
                const float xc = silu_fast(acc);
                win = make_float4(win.y, win.z, xv[j], 0.f);
                if ((smask >> n) & 1u) __stcs(&cs[(n / TB) * cst], win);
                put_b(buf, n, e, xc);
                xv[j] = xc;
              }
              tc::tmem_st8(tq + col, xv);                   // the scan reads xc here (the hi-operand columns)
            }
          }
          tc::tmem_wait_st();
          gemm_done(2 * LT_E);                              // z tiles too, before the next GEMM's wait
          push_slices(buf, (int)rank * (LT_E * 128 / PER), LT_E * 128 / PER);   // xc: x_proj runs whole
        }
        arrive_act();
        mark(PF_CONV);
        if (!(ok = wait_mma())) break;
        mark(PF_W_XP);
        // ---- x_proj epilogue: dt_r -> operand (K slice 0, zero padded), B/C -> smem
        {
          uint8_t* buf = bnext();
          if (g == 0) {
#pragma unroll 1
            for (int gi = 0; gi < NG; ++gi) {
              float v[8], v2[8];
              ldv8((uint32_t)(COL_XP + 8 * gi), v);          // K half 0
              ldv8((uint32_t)(COL_XP + CT + 8 * gi), v2);    // K half 1
#pragma unroll
              for (int j = 0; j < 8; ++j) v[j] += v2[j];
              if (row < DBC) {
#pragma unroll
                for (int j = 0; j < 8; ++j) dbc[(8 * gi + j) * 64 + row] = v[j];
              }
              if (row < PER) {
#pragma unroll
                for (int j = 0; j < 8; ++j) put_b(buf, 8 * gi + j, row, row < R ? v[j] : 0.f);
              }
            }
          }
        }
        arrive_act();
        mark(PF_XP);
        if (!(ok = wait_mma())) break;
        mark(PF_W_DT);
        // ---- selective scan + D skip + SiLU(z) gate, thread per own channel
        //      and chunk run; the next chunk's state loads while one computes
        {
          uint8_t* buf = bnext();
          for (int u = g; u < LT_E * RUNS; u += 4) {
            const int lt = u / RUNS, n0 = (u % RUNS) * RUN;
            const int e = (int)(rank * LT_E + lt) * 128 + row;
            const float4* A2p = reinterpret_cast<const float4*>(lp + LP::A2) + e * 4;
            // time blocks run 4x the columns per channel: keep A in registers there
            float4 Areg[TB > 1 ? 4 : 1];
            if constexpr (TB > 1) {
#pragma unroll
              for (int k = 0; k < 4; ++k) Areg[k] = __ldg(A2p + k);
            }
            const float Dp = __ldg(lp + LP::Dp + e);
            const float bdt = __ldg(lp + LP::dtb + e);
            // SSM state layout [chunk][layer][k = 0..3][channel] of float4: a
            // warp's access for one k is 512 contiguous bytes.  The state is
            // read and written once per step and far larger than L2: loads and
            // stores carry the streaming cache hint (.cs) so they do not evict
            // the weight tiles.
            float4* ss = a.ssm_state + ((long long)c0 * L + l) * 4 * E + e;   // chunk stride 4*L*E
            const long long cstride = (long long)L * 4 * E;
            float4 nx[4];                                   // state of the next chunk, loaded one chunk ahead
#pragma unroll
            for (int k = 0; k < 4; ++k)
              nx[k] = ((lmask >> n0) & 1u) ? __ldcs(&ss[(n0 / TB) * cstride + k * E]) : make_float4(0.f, 0.f, 0.f, 0.f);
            float h[16];
#pragma unroll 1
            for (int gi = 0; gi < RUN / 4; ++gi) {
              const int nb = n0 + 4 * gi;
              float xc[4], z[4], dtr[4];
              tc::tmem_ld4(tq + (uint32_t)(COL_X + lt * CT + nb), xc);   // xc as the conv stored it
              ldv4((uint32_t)(COL_Z + lt * CT + nb), z);
              ldv4((uint32_t)(COL_DT + lt * CT + nb), dtr);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const int n = nb + j;
                if (n % TB == 0) {                          // first position of a chunk: take its state
#pragma unroll
                  for (int k = 0; k < 4; ++k) {
                    h[4 * k] = nx[k].x; h[4 * k + 1] = nx[k].y; h[4 * k + 2] = nx[k].z; h[4 * k + 3] = nx[k].w;
                  }
                  if (n + TB < n0 + RUN) {
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                      nx[k] = ((lmask >> (n + TB)) & 1u) ? __ldcs(&ss[((n + TB) / TB) * cstride + k * E])
                                                         : make_float4(0.f, 0.f, 0.f, 0.f);
                  }
                }
                const float dtv = softplus_f(dtr[j] + bdt);
                const float dx = dtv * xc[j];
                const float4* bc4 = reinterpret_cast<const float4*>(dbc + n * 64 + R);
                float y = 0.f;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                  float4 A4;
                  if constexpr (TB > 1) A4 = Areg[k];
                  else A4 = __ldg(A2p + k);
                  const float4 B4 = bc4[k];
                  const float4 C4 = bc4[4 + k];
                  h[4 * k + 0] = fmaf(h[4 * k + 0], ex2_approx(dtv * A4.x), dx * B4.x);
                  h[4 * k + 1] = fmaf(h[4 * k + 1], ex2_approx(dtv * A4.y), dx * B4.y);
                  h[4 * k + 2] = fmaf(h[4 * k + 2], ex2_approx(dtv * A4.z), dx * B4.z);
                  h[4 * k + 3] = fmaf(h[4 * k + 3], ex2_approx(dtv * A4.w), dx * B4.w);
                  y = fmaf(h[4 * k + 0], C4.x, y);
                  y = fmaf(h[4 * k + 1], C4.y, y);
                  y = fmaf(h[4 * k + 2], C4.z, y);
                  y = fmaf(h[4 * k + 3], C4.w, y);
                }
                if ((smask >> n) & 1u) {
#pragma unroll
                  for (int k = 0; k < 4; ++k)
                    __stcs(&ss[(n / TB) * cstride + k * E], make_float4(h[4 * k], h[4 * k + 1], h[4 * k + 2], h[4 * k + 3]));
                }
                y = fmaf(Dp, xc[j], y);
                y *= silu_fast(z[j]);
                put_b(buf, n, e, y);
              }
            }
          }
          push_slices(buf, (int)rank * (LT_E * 128 / PER), LT_E * 128 / PER);
        }
        arrive_act();
        mark(PF_SCAN);
        if (!(ok = wait_mma())) break;
        mark(PF_W_OUT);
        // ---- out_proj epilogue (own features) -> both CTAs' scratch, then LN2
        for (int u = g; u < LT_D * NG; u += 4) {
          const int lt = u / NG, gi = u % NG;
          const int f = (int)(rank * LT_D + lt) * 128 + row;
          float v[8];
          ldv8((uint32_t)(lt * CT + 8 * gi), v);
          if (f < D) {
#pragma unroll
            for (int j = 0; j < 8; ++j) scr[(8 * gi + j) * D + f] = v[j];
          }
        }
        push_rows(scr, peer_scr, D, (int)rank * LT_D * 128, LT_D * 128);
        if (!(ok = exchange())) break;
        layernorm_to_b(scr, lp + LP::ln2w, lp + LP::ln2b);
        arrive_act();
        mark(PF_LN2);
        mark(PF_W_FF1);
        // ---- ff.0 epilogue (own features): + b1, exact GELU -> both operands.
        //      Units start on finished ff.0 tiles.  With one buffer the GELU
        //      output of tiles below kSafeTile would land on the K slices of
        //      ff.0's own operand, which later tiles still read: those run
        //      after the whole GEMM.
        {
          uint8_t* buf = bnext();
          auto gelu_unit = [&](int u) {
            const int lt = u / NG, gi = u % NG;
            const int f = (int)(rank * LT_F + lt) * 128 + row;
            const float b = __ldg(lp + LP::b1 + f);
            float v[8];
            ldv8((uint32_t)(lt * CT + 8 * gi), v);
#pragma unroll
            for (int j = 0; j < 8; ++j) put_b(buf, 8 * gi + j, f, gelu_f(v[j] + b));
          };
          if constexpr (kSafeTile == 0) {
            for (int u = g; u < LT_F * NG; u += 4) {
              wait_tile(u / NG);                          // ff.0 tile u / NG
              gelu_unit(u);
            }
            gemm_done(LT_F);
          } else {
            for (int u = kSafeTile * NG + g; u < LT_F * NG; u += 4) {
              wait_tile(u / NG);
              gelu_unit(u);
            }
            gemm_done(LT_F);
            for (int u = g; u < kSafeTile * NG; u += 4) gelu_unit(u);
          }
          push_slices(buf, (int)rank * (LT_F * 128 / PER), LT_F * 128 / PER);
        }
        arrive_act();
        mark(PF_FF1);
        if (!(ok = wait_mma())) break;
        mark(PF_W_FF2);
        // ---- ff.2 epilogue (own features): residual update in both CTAs
        for (int u = g; u < LT_D * NG; u += 4) {
          const int lt = u / NG, gi = u % NG;
          const int f = (int)(rank * LT_D + lt) * 128 + row;
          float v[8];
          ldv8((uint32_t)(lt * CT + 8 * gi), v);
          if (f < D) {
            const float b = __ldg(lp + LP::b2 + f);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const int idx = (8 * gi + j) * D + f;
              hres[idx] = hres[idx] + v[j] + b;
            }
          }
        }
        push_rows(hres, peer_hres, D, (int)rank * LT_D * 128, LT_D * 128);
        if (!(ok = exchange())) break;
        mark(PF_FF2);
      }
      if (!ok) break;
      // ---- head.0: Linear + ReLU (own features -> both operands)
      {
        uint8_t* buf = bnext();
        for (int i = ct; i < VC * D; i += kComputeThreads) {
          const int n = i / D, f = i - (i / D) * D;
          put_b(buf, n, f, hres[i]);
        }
      }
      arrive_act();
      mark(PF_HEAD0);
      if (!(ok = wait_mma())) break;
      mark(PF_W_H0);
      {
        uint8_t* buf = bnext();
        for (int u = g; u < LT_D * NG; u += 4) {
          const int lt = u / NG, gi = u % NG;
          const int f = (int)(rank * LT_D + lt) * 128 + row;
          float v[8];
          ldv8((uint32_t)(lt * CT + 8 * gi), v);
          if (f < D) {
            const float b = __ldg(P + o_bh0 + f);
#pragma unroll
            for (int j = 0; j < 8; ++j) put_b(buf, 8 * gi + j, f, fmaxf(v[j] + b, 0.f));
          }
        }
        push_slices(buf, (int)rank * (LT_D * 128 / PER), LT_D * 128 / PER);
      }
      arrive_act();
      mark(PF_HEAD1);
      if (!(ok = wait_mma())) break;
      mark(PF_W_H2);
      // ---- head.2: logits (own vocab half) -> both CTAs' scratch
      for (int u = g; u < LT_V * NG; u += 4) {
        const int lt = u / NG, gi = u % NG;
        const int vv = (int)(rank * LT_V + lt) * 128 + row;
        const float b = __ldg(P + o_bh2 + vv);
        float v[8];
        ldv8((uint32_t)(lt * CT + 8 * gi), v);
#pragma unroll
        for (int j = 0; j < 8; ++j) scr[(8 * gi + j) * 256 + vv] = v[j] + b;
      }
      push_rows(scr, peer_scr, 256, (int)rank * LT_V * 128, LT_V * 128);
      if (!(ok = exchange())) break;
      mark(PF_HEAD2);
      // ---- quantiser + range coder, a warp per chunk (both CTAs, identical);
      //      a chunk's TB positions are coded in order
      for (int ch = cw; ch < CHUNKS; ch += 16)
#pragma unroll 1
      for (int jj = 0; jj < TB; ++jj) {
        const int n = ch * TB + jj;
        const int c = c0 + ch;
        const int t = t0 + jj;                             // position predicted / coded by column n
        if (!((amask >> n) & 1u)) continue;
        if (mode == MODE_LOGITS) {
          if (writer) {
            float* dst = a.logits + ((long long)c * a.n_steps + t) * V;
            for (int v = lane; v < V; v += 32) dst[v] = scr[n * 256 + v];
          }
          if (lane == 0) {
            const int nt = t + TB;                         // this column's position in the next step
            const int nx = (nt < a.n_steps) ? a.tokens[(long long)c * a.n_steps + nt] : 0;
            prev[n] = (nx >= 0 && nx < V) ? nx : 0;
          }
          continue;
        }
        float lv[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) lv[k] = scr[n * 256 + lane * 8 + k];
        uint32_t fr[8], base;
        bq_quantise_warp<8>(lv, V, a.precision, lane, fr, base);
        if (mode == MODE_ENCODE) {
          int sym = a.bytes[(long long)c * a.in_pitch + (t - origin)];
          if (sym >= V) {
            if (lane == 0 && writer) atomicOr(a.err, RC_ERR_SYMBOL);
            sym = 0;
          }
          uint32_t left, freq;
          bq_lookup_warp<8>(fr, base, sym, lane, left, freq);
          if (lane == 0) {
            RcEnc st = encs[n / TB];
            if (writer) {
              rc_enc_put(st, left, freq, a.precision, a.words + (long long)c * a.pitch_words, a.pitch_words, a.err);
              encs[n / TB] = st;
            }
            if constexpr (TB == 1) {
              prev[n] = sym;
            } else {                                       // input of this column in the next step
              const int nt = t + TB - 1;
              const int nx = nt < lens_sh[n] ? a.bytes[(long long)c * a.in_pitch + (nt - origin)] : 0;
              prev[n] = nx < V ? nx : 0;
            }
          }
        } else if constexpr (TB == 1) {
          RcDec st = decs[n];
          unsigned long long scale;
          const uint32_t target = rc_dec_target(st, a.precision, scale);
          uint32_t left, freq;
          const int sym = bq_search_warp<8>(fr, base, target, lane, left, freq);
          if (lane == 0) {
            int nw = a.sizes_in[c];
            nw = nw < 0 ? 0 : (nw > a.pitch_words ? a.pitch_words : nw);
            rc_dec_advance(st, scale, left, freq, a.words_in + (long long)c * a.pitch_words, nw);
            decs[n] = st;
            if (writer) a.out[(long long)c * a.out_pitch + (t - origin)] = (uint8_t)sym;
            prev[n] = sym;
          }
        }
      }
      if constexpr (HL == 4) {
        if (__any_sync(0xffffffffu, range_bad) && lane == 0) atomicOr(a.err, RC_ERR_RANGE);
        range_bad = false;
      }
      cbar_sync();
      mark(PF_CODER);
    }
#ifdef BOA_PHASE_PROFILE
    if (pon) for (int i = 0; i < 20; ++i) a.prof[i] = pacc[i];
#endif
    if (ok && mode == MODE_ENCODE && ct < CHUNKS && writer) {
      const int c = c0 + ct;
      if (c < a.n_chunks) {
        RcEnc st = encs[ct];
        a.sizes[c] = rc_enc_finish(st, a.words + (long long)c * a.pitch_words, a.pitch_words, a.err);
      }
    }
  }

  // ------------------------------ teardown ------------------------------
  tc::tc_fence_before();
  __syncthreads();
  if (tid == 0 && *abort_flag) {
    atomicOr(a.err, RC_ERR_TIMEOUT);
    // weight copies still in flight must land before the CTA exits: the
    // newest copy issued into each ring slot is the only one that can be
    for (int sj = 0; sj < kStagesK; ++sj) {
      if (slot_ph[sj] == 0xffu) continue;
      const long long t0 = clock64();
      while (!tc::mbar_try_wait(&full[sj], (uint32_t)slot_ph[sj])) {
        if (clock64() - t0 > kWaitBudget) break;
      }
    }
  }
  __syncthreads();
  // neither CTA of a pair may exit while the peer can still write into it
  if constexpr (SPLIT == 2) cluster_sync_all();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

}  // namespace boa

// The device model: everything the launch helpers need.
struct boa_model {
  int D, L, V, kind, device;
  int n_sms = 148;
  boa::TilePlan plan;         // split 1
  boa::TilePlan plan2;        // split 2 (valid when has_split2)
  bool has_split2 = false;
  uint8_t* d_tiles = nullptr;     // split-1 stream
  uint8_t* d_tiles2 = nullptr;    // split-2 streams, rank 0 then rank 1
  float* d_params = nullptr;
  uint32_t* d_err = nullptr;      // device-side error bits of the calls on this model
  size_t params_floats = 0;
  int time_block = 0;             // positions per step in encode / logits mode: 0 (choose 4 or 8), 1, 4 or 8
};

namespace boa {

template <int D, int KIND, int CT, int SPLIT, int TB = 1>
int launch_step_ct(StepArgs& a, int n_chunks, cudaStream_t s) {
  constexpr int VC = CT / tc::OpKind<KIND>::kHiLo;
  const int smem = Smem<D, KIND, CT, SPLIT>::ALLOC;
  auto kern = k_boa_step<D, KIND, CT, SPLIT, TB>;
  // The warpgroups' setmaxnreg shares add up to kRegsLaunch registers a thread
  // at launch; with fewer the compute warps' increase could never be granted.
  static const int launch_regs = [&] {
    cudaFuncAttributes fa{};
    return cudaFuncGetAttributes(&fa, kern) == cudaSuccess ? fa.numRegs : -1;
  }();
  if (launch_regs != kRegsLaunch)
    return boa_fail(BOA_ERR_UNSUPPORTED, "k_boa_step: unexpected register allocation for the warpgroup split");
  BOA_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  const int grid = cdiv(n_chunks, VC / TB) * SPLIT;
  if constexpr (SPLIT == 1) {
    kern<<<grid, threads_for(SPLIT), smem, s>>>(a);
  } else {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(threads_for(SPLIT), 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = SPLIT;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    BOA_CUDA(cudaLaunchKernelEx(&cfg, kern, a));
  }
  BOA_CUDA(cudaGetLastError());
  return BOA_OK;
}

// Time blocks of 8 positions need chunk runs of whole blocks in the scan.
template <int D, int KIND>
constexpr bool time_block8_ok() {
  constexpr int VC = ChunkTileMax<D, KIND>::value / tc::OpKind<KIND>::kHiLo;
  constexpr int LT_E = 2 * D / 128;
  return (VC / (LT_E >= 4 ? 1 : 4 / LT_E)) % 8 == 0;
}

// Time block of an encode / logits run when the model leaves the choice open:
// 8 when the launch then takes less time than with 4, estimated as (waves of
// CTAs, one per SM) x (kernel steps + a CTA's start-up, about 6 steps).  Both
// cost about the same per step, but 8 halves the steps and doubles the CTAs,
// which fills the last wave better (1000 chunks of 2xFP16 at d_model 256:
// 7 waves x 512 steps instead of 4 x 1024 per 4096 positions; encode about
// 17 % faster) and halves the steps of one-wave launches.
inline int choose_time_block(int n_chunks, int chunks_per_cta_tb1, int positions, int n_sms) {
  constexpr int kStartSteps = 6;
  const auto cost = [&](int tb) {
    const long long ctas = cdiv(n_chunks, chunks_per_cta_tb1 / tb);
    return (long long)cdiv((int)ctas, n_sms) * (cdiv(positions, tb) + kStartSteps);
  };
  return positions >= 8 && cost(8) < cost(4) ? 8 : 4;
}

// Positions per kernel step of an encode / logits launch over n_chunks chunks
// and `positions` positions (1: one position per step).
template <int D, int KIND>
int encode_time_block_t(const boa_model* m, int n_chunks, int positions) {
  if (m->time_block == 1 || positions < 4) return 1;
  if constexpr (time_block8_ok<D, KIND>()) {
    if (m->time_block == 0)
      return choose_time_block(n_chunks, ChunkTileMax<D, KIND>::value / tc::OpKind<KIND>::kHiLo, positions,
                               m->n_sms);
    return m->time_block == 8 && positions >= 8 ? 8 : 4;
  }
  return 4;
}

// Pick the decomposition.  Encode and logits runs of at least 4 positions use
// time blocks of 4 or 8 positions (choose_time_block, or the model's setting)
// on the widest single-CTA tile (32 operand columns: 8 chunks with 16-bit
// operands at d_model <= 256, 8 value columns with 2xFP16, 16 with 3xTF32,
// else 16 columns).  Decode, and single steps, use one
// position per step: clusters of two CTAs (half the features each) when
// 16-chunk tiles would leave SMs idle, 32-column tiles when there are chunks
// enough to fill every SM, 16-column single CTAs otherwise (the split kind at
// d_model 64 always takes 32 columns: its scan needs 16 value columns).  Every
// choice gives the same per-column arithmetic.
template <int D, int KIND>
int launch_step_t(const boa_model* m, StepArgs& a, int n_chunks, cudaStream_t s, int positions) {
  constexpr int HL = tc::OpKind<KIND>::kHiLo;
  const bool blocked = a.mode == MODE_ENCODE || a.mode == MODE_LOGITS;
  const int tb = blocked ? encode_time_block_t<D, KIND>(m, n_chunks, positions) : 1;
  if (tb > 1) {
    a.tiles_per_step = m->plan.per_step;
    a.tiles_per_layer = m->plan.per_layer;
    a.wtiles = m->d_tiles;
    constexpr int CTM = ChunkTileMax<D, KIND>::value;
    if constexpr (time_block8_ok<D, KIND>()) {
      if (tb == 8) return launch_step_ct<D, KIND, CTM, 1, 8>(a, n_chunks, s);
    }
    return launch_step_ct<D, KIND, CTM, 1, 4>(a, n_chunks, s);
  }
  if constexpr (D == 256 && (KIND == 1 || KIND == 2)) {
    if (m->has_split2 && 2 * cdiv(n_chunks, 16) <= m->n_sms) {
      a.tiles_per_step = m->plan2.per_step;
      a.tiles_per_layer = m->plan2.per_layer;
      a.wtiles = m->d_tiles2;
      return launch_step_ct<D, KIND, 16, 2>(a, n_chunks, s);
    }
  }
  a.tiles_per_step = m->plan.per_step;
  a.tiles_per_layer = m->plan.per_layer;
  a.wtiles = m->d_tiles;
  if constexpr (HL >= 2 && D == 64) {
    return launch_step_ct<D, KIND, ChunkTileMax<D, KIND>::value, 1>(a, n_chunks, s);
  } else if constexpr (HL == 4) {
    return launch_step_ct<D, KIND, 32, 1>(a, n_chunks, s);      // 8 value columns, MMA N = 16
  } else {
    if constexpr (ChunkTileMax<D, KIND>::value == 32) {
      if (n_chunks >= (32 / HL) * m->n_sms) return launch_step_ct<D, KIND, 32, 1>(a, n_chunks, s);
    }
    return launch_step_ct<D, KIND, 16, 1>(a, n_chunks, s);
  }
}

// Explicit instantiations, one translation unit per operand kind.
#define BOA_DECLARE_LAUNCH(DD, KK) \
  extern template int launch_step_t<DD, KK>(const boa_model*, StepArgs&, int, cudaStream_t, int);
#define BOA_DEFINE_LAUNCH(DD, KK) \
  template int launch_step_t<DD, KK>(const boa_model*, StepArgs&, int, cudaStream_t, int);

BOA_DECLARE_LAUNCH(64, 0)
BOA_DECLARE_LAUNCH(256, 0)
BOA_DECLARE_LAUNCH(64, 1)
BOA_DECLARE_LAUNCH(256, 1)
BOA_DECLARE_LAUNCH(512, 1)
BOA_DECLARE_LAUNCH(64, 2)
BOA_DECLARE_LAUNCH(256, 2)
BOA_DECLARE_LAUNCH(512, 2)
BOA_DECLARE_LAUNCH(64, 3)
BOA_DECLARE_LAUNCH(256, 3)
BOA_DECLARE_LAUNCH(64, 4)
BOA_DECLARE_LAUNCH(256, 4)

}  // namespace boa
