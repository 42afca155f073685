// NVFP4 block-scaled GEMM kernels for sm_100a (B200).
//
// One persistent, warp-specialised kernel body serves both the dense GEMM
// (kernels/gemm/submission.py:51-583 in the reference) and the grouped GEMM
// (kernels/group_gemm/submission.py:55-703).  It computes
//
//     D[p, q] = sum_k  e2m1(P[p, k]) * sfP[p, k/16]  *  e2m1(Q[q, k]) * sfQ[q, k/16]
//
// with fp32 accumulation in tensor memory and stores fp16.  P is the operand
// on the 128-row MMA M side, Q the operand on the MMA N side (BN rows).  For
// the ordinary order P = A (M rows), Q = B (N rows) and C[m, n] = D[m, n]; for
// "swap" P = B, Q = A and C[m, n] = D[n, m], which puts a skinny M (decode-like
// shapes, small MoE groups) on the flexible N side of the MMA.
//
// Roles (20 warps):
//   warps 0-7   epilogue: warp w drains TMEM lanes 32*(w%4).. and column half w/4 of the
//               accumulator into registers as fp16 (two 32-column chunks at a time),
//               releases the accumulator after its last load, and stores C with TMA through
//               small shared-memory staging buffers while the next tile's MMAs already run
//   warps 8-10  producers (k-steps round-robin): TMA loads of the P and Q tiles (128-byte
//               swizzle) into a ring of kStages stages
//   warp 11     TMEM owner and MMA issuer: per k-step it waits for the stage's operand
//               tiles (full) and its scales in TMEM (sf_full), issues tcgen05.mma
//               kind::mxf4nvf4 (K = 64 per instruction) and two tcgen05.commits (the stage,
//               the TMEM scale buffer)
//   warps 12-19 scale warps, two groups of four (group g serves k-steps j with j % 2 == g):
//               the group loads its steps' scale atoms into its own shared-memory slots
//               (dense: tensor loads through 8-byte-element scale maps; grouped: plain bulk
//               copies), and each warp moves them into its own 32 TMEM lanes with ld.shared +
//               tcgen05.st once the step's TMEM scale buffer is free.  tcgen05.cp would run
//               in the MMA's own queue (~56 cycles per 512-byte atom, not overlapped with the
//               MMAs), register stores run alongside them.
//   CTA pairs (cta_group::2, M = 256): the leader issues the MMAs; both CTAs' tensor loads
//   count on the leader's full barrier and both CTAs' scale warps arrive on its sf_full.
//
// Scale factors arrive in the reference's pre-permuted layout
// (kernels/gemm/reference.py:113-150): per 128-row block and per 64-wide K block
// one 512-byte atom whose byte (r % 32) * 16 + (r / 32) * 4 + j holds row r,
// K-vector j.  The four atoms of one 256-wide K stage are contiguous (2 KiB) and
// arrive with one bulk copy.  The MMA reads the scales of row r from TMEM column
// (r / 32), lane (r % 32) of every lane quarter, so every scale warp stores atom
// row `lane` (16 bytes = 4 columns) into its own quarter: the same bytes land in
// all four quarters.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include "ptx_sm100.cuh"

namespace nvfp4 {

constexpr int kBM = 128;            // MMA M (rows of P per tile)
constexpr int kAtomBytes = 512;     // one scale-factor atom: 128 rows x 4 K-vectors
constexpr int kEpiWarps = 8;
// Producer warps 8..10 take the k-steps round-robin: a TMA instruction occupies its issuing
// thread for ~160 cycles, so one thread issues a stage (2 tensor + up to 3 bulk copies)
// only every ~0.4 us.
constexpr int kProducerWarp = 8;
constexpr int kNumProducers = 3;  // (a 21st warp would cost the block its 96-register budget)
constexpr int kMmaWarp = kProducerWarp + kNumProducers;
constexpr int kFirstSfWarp = kMmaWarp + 1;
constexpr int kSfGroups = 2;        // groups of 4 scale warps; group g serves k-steps j % 2 == g
constexpr int kNumThreads = 32 * (kFirstSfWarp + 4 * kSfGroups);
constexpr int kMaxDynamicSmem = 232448;     // opt-in dynamic shared memory per CTA on sm_100

// KB = 64-wide K blocks per pipeline stage: 4 (256 K, one 128-byte swizzle row per
// operand row) or 2 (128 K, 64-byte swizzle).  Smaller stages fit twice as many in
// shared memory, so stages are released and refilled at half the granularity.
template <int BN, int KB, bool CTA2 = false>
struct Cfg {
  static_assert(BN == 64 || BN == 128 || BN == 192 || BN == 256, "BN must be 64, 128, 192 or 256");
  static_assert(KB == 2 || KB == 4, "KB must be 2 or 4");
  static constexpr int kBKBytes = KB * 32;            // bytes of K per stage per row
  static constexpr int kBK = KB * 64;                 // K elements per stage
  static constexpr uint32_t kSwizzle = KB == 4 ? 2 : 4;  // smem descriptor: 128B / 64B swizzle
  static constexpr uint32_t kSbo = 8 * kBKBytes;      // bytes between 8-row core-matrix groups
  static constexpr int kPBytes = kBM * kBKBytes;
  static constexpr int kQRows = CTA2 ? BN / 2 : BN;  // Q rows this CTA stages (the pair splits N)
  static constexpr int kQBytes = kQRows * kBKBytes;
  static constexpr int kSfqAtoms = (BN <= 128) ? 1 : 2;  // 128-row scale blocks per Q tile
  static constexpr int kSfpBytes = KB * kAtomBytes;
  static constexpr int kSfqBytes = kSfqAtoms * KB * kAtomBytes;
  static constexpr int kStageBytes = kPBytes + kQBytes;       // operand tiles of one k-step
  static constexpr int kSfSlotBytes = kSfpBytes + kSfqBytes;  // scale atoms of one k-step
  static constexpr int kSfqColsPerKb = 4 * kSfqAtoms;
  // TMEM columns of one scale buffer: [SFP kb0..kb(KB-1) (4 columns each)][SFQ kb0..]
  static constexpr int kSfpCols = 4 * KB;
  static constexpr int kSfCols = kSfpCols + KB * kSfqColsPerKb;
  static constexpr int kAccStages = (BN <= 128) ? 2 : 1;
  // TMEM scale buffers: a ring of its own (kSfBufs deep), next to the accumulators.  The
  // scales of step j go into buffer j % kSfBufs once the MMAs of step j - kSfBufs are done.
  static constexpr int kSfBufsRaw = (512 - kAccStages * BN) / kSfCols;
  static constexpr int kSfBufs = kSfBufsRaw > 8 ? 8 : kSfBufsRaw;
  // Shared memory: [operand stages][epilogue staging][scale slots][barriers].
  //
  // Scale atoms travel in their own ring of NS shared-memory slots (even: slot j % NS is
  // always served by the scale-warp group of step j, which loads it itself).  Operand stages
  // first, as many as fit beside kMinSlots slots and 8 KB of epilogue staging (cap 8); then
  // up to 8 slots in what is left.
  static constexpr int kMinSlots = 4;
  static constexpr int kAvail = kMaxDynamicSmem - 1024 /* base alignment */ - 512 /* barriers */;
  static constexpr int kStagesRaw = (kAvail - kMinSlots * kSfSlotBytes - 8192) / kStageBytes;
  static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
  static constexpr int kSfSlotsRaw = (kAvail - kStages * kStageBytes - 8192) / kSfSlotBytes;
  static constexpr int kSfSlots = kSfSlotsRaw >= 8 ? 8 : (kSfSlotsRaw & ~1);
  // Epilogue staging for the TMA stores of C: per epilogue warp kEpiBufs buffers of 1 KB
  // (32 rows x 16 fp16 columns of C; 16 rows x 32 columns in the swapped order), two
  // (double buffering) where they fit.
  static constexpr int kRest = kAvail - kStages * kStageBytes - kSfSlots * kSfSlotBytes;
  static constexpr int kEpiBufs = kRest >= 2 * kEpiWarps * 1024 ? 2 : 1;
  static constexpr int kEpiBytes = kEpiBufs * kEpiWarps * 1024;
  static constexpr int kColsNeeded = kAccStages * BN + kSfBufs * kSfCols;
  static constexpr int kTmemCols = kColsNeeded <= 32 ? 32 : kColsNeeded <= 64 ? 64
                                 : kColsNeeded <= 128 ? 128 : kColsNeeded <= 256 ? 256 : 512;
  static constexpr int kSfCol0 = kAccStages * BN;
  // barriers: full[S], empty[S], sf_full[T], sf_empty[T], acc_full[A], acc_empty[A], drain,
  // sf_data[NS], sf_free[NS]
  static constexpr int kNumBars = 2 * kStages + 2 * kSfBufs + 2 * kAccStages + 1 + 2 * kSfSlots;
  static constexpr int kBarrierBytes = 8 * kNumBars + 16;
  static constexpr int kSmemBytes =
      1024 + kStages * kStageBytes + kEpiBytes + kSfSlots * kSfSlotBytes + kBarrierBytes;
  // a producer's previous step j - kNumProducers must imply that step j - 2 S was consumed,
  // or its parity wait on the empty barrier for step j - S could alias
  static_assert(kStages >= kNumProducers, "need at least one stage per producer warp");
  static_assert(kSfBufs >= 2, "TMEM scale ring too shallow");
  static_assert(kSfSlots % kSfGroups == 0 && kSfSlots >= 2 * kSfGroups,
                "each scale slot must belong to one scale-warp group");
  static_assert(kColsNeeded <= 512, "TMEM budget exceeded");
  static_assert(kBarrierBytes <= 512, "barrier area exceeded");
  static_assert(kSmemBytes <= kMaxDynamicSmem, "shared memory budget exceeded");
  static_assert((kStages * kStageBytes) % 1024 == 0, "staging buffers must stay 1 KB aligned");
};

// Everything the kernel needs; tensor maps for the dense case are separate
// __grid_constant__ parameters.
struct GemmParams {
  // dense problem (ignored when grouped)
  int p_rows, q_rows, K, L;
  __half* C;
  long long ldc;                // elements between rows of C
  long long c_batch;            // elements between batches of C
  int tiles_p, tiles_q, total_tiles;
  // raster: bands of band_p P tiles; within a band the P tiles vary fastest, then the Q
  // tiles, so the concurrent tiles share one band of P rows (kept in L2) while Q streams
  int band_p;
  // grouped problem
  int G;
  const int* sizes;             // G x 4: m, n, k, l
  const unsigned long long* abc;  // G x 3: a, b, c
  const unsigned long long* sfs;  // G x 2: sfa (permuted), sfb (permuted)
  const CUtensorMap* maps;      // G x 5: [P operand, Q operand, C_g store, P scales, Q scales]
  const int* tile_prefix;       // G + 1 running tile counts
  // stream-K (dense only): when sk_ktn > 0 every CTA takes an equal contiguous range of
  // the total_tiles x sk_ktn k-steps; partial tiles meet through sk_slots / sk_flags
  int sk_ktn;
  float* sk_slots;              // per CTA: BN/4 x 128 float4 (column group major)
  unsigned* sk_flags;           // per CTA: kSkPublished while its partial is published
  // n_out > 0: store C into outs[0 .. n_out) instead (each already offset to this GEMM's
  // columns, row stride ldc; peers' buffers reached over NVLink with plain stores), L = 1
  int n_out;
  unsigned long long outs[8];
  // dense: 1 = C is stored with TMA (tensor map tm_c; N % 8 == 0, C 16-byte aligned, one
  // output buffer); grouped: decided per group from its n and C address
  int c_tma;
  // fused epilogue (dense): out = act(acc + bias[n]) stored as fp16 or bf16
  const float* bias;            // per output column n, or null
  int act;                      // 0 none, 1 relu, 2 gelu (erf form)
  int out_bf16;                 // 1: C is bf16
  // control
  int* status;
  unsigned long long timeout_ns;
  // Test bit 1: the producers issue nothing, so every pipeline wait runs out (the timeout
  // path's test).  0 in normal use.
  int debug;
};

// Per-tile view shared by all roles.
struct TileInfo {
  int p0, q0, l;
  int p_rows, q_rows, K;
  const void* map_p;
  const void* map_q;
  const void* map_c;     // C store map (TMA epilogue)
  const void* map_sfp;   // scale maps of P and Q (8-byte elements: row = 128-row block)
  const void* map_sfq;
  bool c_tma;
  __half* C;             // batch-adjusted base
  long long ldc;
  int rk;                // 64-wide K blocks (atoms per 128-row block)
  int num_kt;            // K stages (KB * 64 wide)
};

constexpr unsigned kSkPublished = 0x9E3779B9u;  // stream-K flag value of a published partial

// A CTA's work is a list of segments: k-steps [kt0, kt1) of tile t (kt1 is clipped to the
// tile's k-steps).  Without stream-K a segment is a whole tile, CTA w taking tiles w,
// w + step, ...; with stream-K CTA w takes global k-steps [start(w), start(w + 1)) of the
// tiles laid end to end, which is at most a tail, whole tiles and a head.
struct Seg {
  int t, kt0, kt1;
};
__device__ __forceinline__ int sk_start(const GemmParams& prm, int w, int nwork) {
  return (int)((long long)prm.total_tiles * prm.sk_ktn * w / nwork);
}
template <bool SK>
__device__ __forceinline__ bool seg_first(const GemmParams& prm, int total, int w, int step, Seg& sg) {
  if constexpr (SK) {
    const int b = sk_start(prm, w, step), e = sk_start(prm, w + 1, step);
    if (b >= e) return false;
    sg.t = b / prm.sk_ktn;
    sg.kt0 = b - sg.t * prm.sk_ktn;
    sg.kt1 = min(prm.sk_ktn, e - sg.t * prm.sk_ktn);
    return true;
  }
  sg.t = w;
  sg.kt0 = 0;
  sg.kt1 = 0x7fffffff;
  return w < total;
}
template <bool SK>
__device__ __forceinline__ bool seg_next(const GemmParams& prm, int total, int w, int step, Seg& sg) {
  if constexpr (SK) {
    const int e = sk_start(prm, w + 1, step);
    sg.t += 1;
    if (sg.t * prm.sk_ktn >= e) return false;
    sg.kt0 = 0;
    sg.kt1 = min(prm.sk_ktn, e - sg.t * prm.sk_ktn);
    return true;
  }
  sg.t += step;
  return sg.t < total;
}

template <bool GROUPED, bool SWAP, int BN, int KB, bool CTA2 = false>
__device__ __forceinline__ bool decode_tile(const GemmParams& prm, const CUtensorMap* tm_p,
                                            const CUtensorMap* tm_q, const CUtensorMap* tm_c,
                                            const CUtensorMap* tm_sfp, const CUtensorMap* tm_sfq, int t,
                                            TileInfo& ti) {
  if constexpr (!GROUPED) {
    const int per_batch = prm.tiles_p * prm.tiles_q;
    const int l = t / per_batch;
    const int r = t - l * per_batch;
    int pb, qb;
    const int per_band = prm.band_p * prm.tiles_q;
    const int band = r / per_band;
    const int rb = r - band * per_band;
    const int p_first = band * prm.band_p;
    const int gb = min(prm.band_p, prm.tiles_p - p_first);
    pb = p_first + rb % gb;
    qb = rb / gb;
    // a CTA pair covers 256 P rows; this CTA owns rows [p0, p0 + 128)
    ti.p0 = CTA2 ? pb * 2 * kBM + (int)cluster_ctarank() * kBM : pb * kBM;
    ti.q0 = qb * BN;
    ti.l = l;
    ti.p_rows = prm.p_rows;
    ti.q_rows = prm.q_rows;
    ti.K = prm.K;
    ti.map_p = tm_p;
    ti.map_q = tm_q;
    ti.map_c = tm_c;
    ti.map_sfp = tm_sfp;
    ti.map_sfq = tm_sfq;
    ti.c_tma = prm.c_tma != 0;
    ti.C = prm.C + (long long)l * prm.c_batch;
    ti.ldc = prm.ldc;
    ti.rk = (prm.K + 63) / 64;
    ti.num_kt = (prm.K + KB * 64 - 1) / (KB * 64);
    return true;
  } else {
    // binary search the group whose tile range holds t
    int lo = 0, hi = prm.G - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (__ldg(prm.tile_prefix + mid) <= t) lo = mid; else hi = mid - 1;
    }
    const int g = lo;
    const int m = __ldg(prm.sizes + 4 * g + 0);
    const int n = __ldg(prm.sizes + 4 * g + 1);
    const int k = __ldg(prm.sizes + 4 * g + 2);
    const int r = t - __ldg(prm.tile_prefix + g);
    // swapped: P = B_g (n rows), Q = A_g (m token rows); otherwise P = A_g, Q = B_g.  The
    // tiles of a group are walked Q first (the concurrent tiles share P rows).
    const int prow = SWAP ? n : m;
    const int qrow = SWAP ? m : n;
    const int tq = (qrow + BN - 1) / BN;
    const int qb = r % tq;
    const int pb = r / tq;
    // a CTA pair covers 256 P rows; this CTA owns rows [p0, p0 + 128)
    ti.p0 = CTA2 ? pb * 2 * kBM + (int)cluster_ctarank() * kBM : pb * kBM;
    ti.q0 = qb * BN;
    ti.l = 0;
    ti.p_rows = prow;
    ti.q_rows = qrow;
    ti.K = k;
    ti.map_p = prm.maps + 5 * g;
    ti.map_q = prm.maps + 5 * g + 1;
    ti.map_c = prm.maps + 5 * g + 2;
    ti.map_sfp = prm.maps + 5 * g + 3;
    ti.map_sfq = prm.maps + 5 * g + 4;
    ti.C = reinterpret_cast<__half*>(__ldg(prm.abc + 3 * g + 2));
    ti.c_tma = (n & 7) == 0 && (reinterpret_cast<uintptr_t>(ti.C) & 15) == 0;
    ti.ldc = n;
    ti.rk = (k + 63) / 64;
    ti.num_kt = (k + KB * 64 - 1) / (KB * 64);
    return true;
  }
}

// Fused epilogue: bias of output column n, activation, then the output type's rounding.
__device__ __forceinline__ float epi_post(const GemmParams& prm, float v, int n, int ncols) {
  if (prm.bias && n < ncols) v += __ldg(prm.bias + n);
  if (prm.act == 1) v = fmaxf(v, 0.f);
  else if (prm.act == 2) v = 0.5f * v * (1.f + erff(v * 0.70710678118654752f));
  return v;
}
__device__ __forceinline__ uint32_t epi_pack(const GemmParams& prm, float x, float y) {
  if (prm.out_bf16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __half2 h = __floats2half2_rn(x, y);
  return *reinterpret_cast<uint32_t*>(&h);
}

// (The F32 and SK instantiations leave parts of the shared epilogue unreachable: the packed
// fp16 loop after the fp32 path's `continue`.)
#pragma nv_diagnostic push
#pragma nv_diag_suppress 128, 177
// SK: stream-K schedule (dense, BN <= 128); F32: fp32 C (dense).  Separate instantiations,
// so that the plain fp16 schedule's code and register allocation are not touched by them.
template <bool GROUPED, bool SWAP, int BN, int KB, bool CTA2 = false, bool SK = false, bool F32 = false>
__global__ void __launch_bounds__(kNumThreads, 1)
nvfp4_gemm_kernel(const __grid_constant__ CUtensorMap tm_p, const __grid_constant__ CUtensorMap tm_q,
                  const __grid_constant__ CUtensorMap tm_sfp, const __grid_constant__ CUtensorMap tm_sfq,
                  const __grid_constant__ CUtensorMap tm_c, const GemmParams prm) {
  static_assert(!SK || (!GROUPED && !CTA2 && BN <= 128), "stream-K: dense, 1-CTA, BN <= 128");
  using C_ = Cfg<BN, KB, CTA2>;
  constexpr int S = C_::kStages;
  constexpr int A = C_::kAccStages;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);

  // [stage 0 .. S-1: P | Q] [epilogue staging] [scale slot 0 .. NS-1: SFP | SFQ atoms]
  // [barriers]
  constexpr int NS = C_::kSfSlots;
  constexpr int T = C_::kSfBufs;
  auto stage_off = [&](int s) { return (uint32_t)(s * C_::kStageBytes); };
  constexpr uint32_t kOffQ = C_::kPBytes;
  constexpr uint32_t kEpi0 = S * C_::kStageBytes;
  constexpr uint32_t kSlot0 = kEpi0 + C_::kEpiBytes;
  auto slot_off = [&](int j) { return kSlot0 + (uint32_t)(j * C_::kSfSlotBytes); };
  constexpr uint32_t kOffSfq = C_::kSfpBytes;  // within a slot
  const uint32_t bar_base = base + kSlot0 + NS * C_::kSfSlotBytes;
  auto full_bar = [&](int s) { return bar_base + 8 * s; };
  auto empty_bar = [&](int s) { return bar_base + 8 * (S + s); };
  auto sff_bar = [&](int t) { return bar_base + 8 * (2 * S + t); };      // scales in TMEM buffer t
  auto sfe_bar = [&](int t) { return bar_base + 8 * (2 * S + T + t); };  // TMEM buffer t free
  auto accf_bar = [&](int a) { return bar_base + 8 * (2 * S + 2 * T + a); };
  auto acce_bar = [&](int a) { return bar_base + 8 * (2 * S + 2 * T + A + a); };
  const uint32_t drain_bar = bar_base + 8 * (2 * S + 2 * T + 2 * A);
  auto sfd_bar = [&](int j) { return bar_base + 8 * (2 * S + 2 * T + 2 * A + 1 + j); };       // slot landed
  auto sfs_bar = [&](int j) { return bar_base + 8 * (2 * S + 2 * T + 2 * A + 1 + NS + j); };  // slot free
  uint8_t* bar_ptr = smem + kSlot0 + NS * C_::kSfSlotBytes;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(bar_ptr + 8 * C_::kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bar_ptr + 8 * C_::kNumBars + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  pdl_launch_dependents();
  // CTA pairs: rank 0 (leader) issues the MMAs for both; tiles are walked per pair.
  const uint32_t crank = CTA2 ? cluster_ctarank() : 0;
  const bool leader = crank == 0;
  const int work0 = CTA2 ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int work_step = CTA2 ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  // arrive on the leader CTA's copy of a barrier (the pair's scale and accumulator hand-offs)
  auto arrive_leader = [&](uint32_t bar) {
    if (CTA2) mbar_arrive_cluster(mapa_shared(bar, 0));
    else mbar_arrive(bar);
  };

  if (threadIdx.x == 0) {
    // one arrive per scale warp of the group serving the stage (of both CTAs of a pair),
    // one per epilogue warp
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int t = 0; t < T; ++t) {
      mbar_init(sff_bar(t), CTA2 ? 8 : 4);
      mbar_init(sfe_bar(t), 1);
    }
    for (int a = 0; a < A; ++a) {
      mbar_init(accf_bar(a), 1);
      mbar_init(acce_bar(a), kEpiWarps * (CTA2 ? 2 : 1));
    }
    mbar_init(drain_bar, 1);
    for (int j = 0; j < NS; ++j) {
      mbar_init(sfd_bar(j), 1);
      mbar_init(sfs_bar(j), 4);  // the 4 scale warps (of this CTA) that moved the slot's atoms
    }
    *abort_flag = 0;
    fence_mbar_init();
    fence_async_shared();
  }
  if (warp >= kProducerWarp && warp < kProducerWarp + kNumProducers && lane == 0 && !GROUPED) {
    prefetch_tmap(&tm_p);
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_sfp);
    prefetch_tmap(&tm_sfq);
    prefetch_tmap(&tm_c);
    // Pull this CTA's first k-stages into L2 while the previous kernel finishes: an L2
    // prefetch is safe before the wait on that kernel even if it writes these inputs
    // (L2 is the point of coherence, nothing lands in this SM).  Dense only: the grouped
    // schedule is itself written by the preceding prep kernel.
    Seg sg0;
    if (seg_first<SK>(prm, prm.total_tiles, work0, work_step, sg0)) {
      TileInfo ti;
      decode_tile<GROUPED, SWAP, BN, KB, CTA2>(prm, &tm_p, &tm_q, &tm_c, &tm_sfp, &tm_sfq, sg0.t, ti);
      const int kte = min(sg0.kt1, ti.num_kt);
      for (int kt = sg0.kt0 + (warp - kProducerWarp); kt < sg0.kt0 + S && kt < kte; kt += kNumProducers) {
        tma_prefetch_l2_3d(&tm_p, kt * C_::kBKBytes, ti.p0, ti.l);
        tma_prefetch_l2_3d(&tm_q, kt * C_::kBKBytes, ti.q0 + (int)crank * C_::kQRows, ti.l);
        tma_prefetch_l2_3d(&tm_sfp, kt * KB * 64, ti.p0 >> 7, ti.l);
        tma_prefetch_l2_3d(&tm_sfq, kt * KB * 64, ti.q0 >> 7, ti.l);
      }
    }
  }
  if (warp == kMmaWarp) {
    if (CTA2) {
      tmem_alloc_2cta(smem_u32(const_cast<uint32_t*>(tmem_slot)), C_::kTmemCols);
      tmem_relinquish_2cta();
    } else {
      tmem_alloc(smem_u32(const_cast<uint32_t*>(tmem_slot)), C_::kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (CTA2) cluster_sync();  // the peer's barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Everything above touches only shared memory, TMEM and kernel parameters, so it
  // overlaps the previous kernel on the stream; global memory is used only after
  // that kernel has completed.
  pdl_wait_prior_grid();
  // (stream-K: the host clears every CTA's flag before the launch)

  const int total = GROUPED ? __ldg(prm.tile_prefix + prm.G) : prm.total_tiles;
  const uint64_t tmo = prm.timeout_ns;
  // scale atoms a Q tile needs (it may start at row 32, 64 or 96 of a 128-row block)
  auto q_atoms = [&](const TileInfo& ti) {
    const int rq = (ti.q_rows + 127) >> 7;
    int nq = ((ti.q0 & 127) + BN + 127) >> 7;
    if (nq > C_::kSfqAtoms) nq = C_::kSfqAtoms;
    if ((ti.q0 >> 7) + nq > rq) nq = rq - (ti.q0 >> 7);
    return nq;
  };
  auto k_blocks = [&](const TileInfo& ti, int kt) {
    const int kbv = ti.rk - kt * KB;
    return kbv > KB ? KB : kbv;
  };

  // Cursor over this CTA's k-steps (tile, k-stage), for the scale loads issued ahead.
  struct Cursor {
    Seg sg;
    int kt, kte;
    bool valid;
    TileInfo ti;
  };
  auto cur_load = [&](Cursor& c) {
    if (!c.valid) return;
    decode_tile<GROUPED, SWAP, BN, KB, CTA2>(prm, &tm_p, &tm_q, &tm_c, &tm_sfp, &tm_sfq, c.sg.t, c.ti);
    c.kt = c.sg.kt0;
    c.kte = min(c.sg.kt1, c.ti.num_kt);
  };
  auto cur_next = [&](Cursor& c) {
    if (++c.kt == c.kte) {
      c.valid = seg_next<SK>(prm, total, work0, work_step, c.sg);
      cur_load(c);
    }
  };

  if (warp >= kProducerWarp && warp < kProducerWarp + kNumProducers) {
    if (lane == 0 && !(prm.debug & 1)) {
      // ------------------------------------------------------------ producers
      // Producer p issues the operand loads of k-steps p, p + 3, ...: one thread issuing TMA
      // copies tops out at about one stage per ~250 ns.
      const uint32_t pid = warp - kProducerWarp;
      uint32_t gstep = 0;
      const uint64_t pol_keep = policy_evict_last();
      int s = 0;
      uint32_t ph = 0;
      const void* last_map = nullptr;
      bool ok = true;
      uint32_t issued_mask = 0, issued_par = 0;
      Seg sg;
      for (bool more = seg_first<SK>(prm, total, work0, work_step, sg); more && ok;
           more = seg_next<SK>(prm, total, work0, work_step, sg)) {
        TileInfo ti;
        decode_tile<GROUPED, SWAP, BN, KB, CTA2>(prm, &tm_p, &tm_q, &tm_c, &tm_sfp, &tm_sfq, sg.t, ti);
        if (GROUPED && ti.map_p != last_map) {
          tmap_fence_acquire(ti.map_p);
          tmap_fence_acquire(ti.map_q);
          last_map = ti.map_p;
        }
        const int kte = min(sg.kt1, ti.num_kt);
        for (int kt = sg.kt0; kt < kte; ++kt, ++gstep) {
          if (gstep % kNumProducers == pid) {
            // stage s free: the MMAs of step gstep - S are done
            if (!mbar_wait_bounded(empty_bar(s), ph ^ 1, abort_flag, prm.status,
                                   kStatusTimeoutProducer, tmo)) { ok = false; break; }
            const uint32_t st = base + stage_off(s);
            if constexpr (CTA2) {
              // both CTAs' tiles count on the leader's full barrier, which the MMA waits on
              if (leader) mbar_arrive_expect_tx(full_bar(s), 2 * (C_::kPBytes + C_::kQBytes));
              const uint32_t fb = mapa_shared(full_bar(s), 0);
              tma_load_3d_pair(st, ti.map_p, fb, kt * C_::kBKBytes, ti.p0, ti.l, pol_keep);
              tma_load_3d_pair(st + kOffQ, ti.map_q, fb, kt * C_::kBKBytes,
                               ti.q0 + (int)crank * C_::kQRows, ti.l, pol_keep);
            } else {
              mbar_arrive_expect_tx(full_bar(s), C_::kPBytes + C_::kQBytes);
              tma_load_3d(st, ti.map_p, full_bar(s), kt * C_::kBKBytes, ti.p0, ti.l, pol_keep);
              tma_load_3d(st + kOffQ, ti.map_q, full_bar(s), kt * C_::kBKBytes,
                          ti.q0 + (int)crank * C_::kQRows, ti.l, pol_keep);
            }
            if (!CTA2 || leader) {  // (a peer cannot wait on the leader's barrier)
              issued_mask |= 1u << s;
              issued_par = (issued_par & ~(1u << s)) | (ph << s);
            }
          }
          if (++s == S) { s = 0; ph ^= 1; }
        }
      }
      if (*abort_flag) {
        // let copies already issued land before the CTA exits (bounded)
        for (int i = 0; i < S; ++i)
          if (issued_mask & (1u << i))
            mbar_wait_plain(full_bar(i), (issued_par >> i) & 1u, 100000000ull);
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0 && leader) {
      // ------------------------------------------------------------ MMA issuer
      bool ok = true;
      int acc = 0;
      uint32_t aph = 0;
      int s = 0;
      uint32_t ph = 0;
      int t = 0;  // TMEM scale buffer
      uint32_t tph = 0;
      Seg sg;
      for (bool more = seg_first<SK>(prm, total, work0, work_step, sg); more && ok;
           more = seg_next<SK>(prm, total, work0, work_step, sg)) {
        TileInfo ti;
        decode_tile<GROUPED, SWAP, BN, KB, CTA2>(prm, &tm_p, &tm_q, &tm_c, &tm_sfp, &tm_sfq, sg.t, ti);
        const int kte = min(sg.kt1, ti.num_kt);
        // A pair splits the instruction's N in halves between the two CTAs' shared memory,
        // so it always issues N = BN (each CTA staged BN/2 rows; rows past the edge are zero).
        int n_mma = ti.q_rows - ti.q0;
        if (n_mma > BN || CTA2) n_mma = BN;
        n_mma = (n_mma + 15) & ~15;
        const uint32_t idesc = make_idesc_mxf4nvf4(CTA2 ? 2 * kBM : kBM, n_mma);
        const uint32_t d_tmem = tmem_base + acc * BN;
        const uint32_t sfq_shift = (ti.q0 & 127) >> 5;
        // (CTA-scope acquire also for the pair's barriers, which the peer arrives on: the
        // data they publish is ordered by the tcgen05 fences and the TMA transaction
        // counts, and a cluster-scope acquire costs ~0.2 us per wait)
        if (!mbar_wait_bounded(acce_bar(acc), aph ^ 1, abort_flag, prm.status, kStatusTimeoutMma,
                               tmo)) { ok = false; break; }
        tc_fence_after();
        for (int kt = sg.kt0; kt < kte; ++kt) {
          // the operand tiles landed (a pair's full barrier counts both CTAs' bytes) and
          // the step's scales are in TMEM buffer t
          if (!mbar_wait_bounded(full_bar(s), ph, abort_flag, prm.status, kStatusTimeoutMma, tmo) ||
              !mbar_wait_bounded(sff_bar(t), tph, abort_flag, prm.status, kStatusTimeoutMma, tmo)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sfp_col = tmem_base + C_::kSfCol0 + t * C_::kSfCols;
          const uint32_t sfq_col = sfp_col + C_::kSfpCols + sfq_shift;
          const uint64_t pdesc = make_smem_desc(base + stage_off(s), 0, C_::kSbo, C_::kSwizzle);
          const uint64_t qdesc = make_smem_desc(base + stage_off(s) + kOffQ, 0, C_::kSbo, C_::kSwizzle);
          const uint32_t acc0 = kt > sg.kt0 ? 1u : 0u;
          if (k_blocks(ti, kt) == KB) {
#pragma unroll
            for (int kb = 0; kb < KB; ++kb) {
              if constexpr (CTA2)
                tc_mma_mxf4nvf4_2cta(d_tmem, pdesc + 2 * kb, qdesc + 2 * kb, idesc, sfp_col + kb * 4,
                                     sfq_col + kb * C_::kSfqColsPerKb, kb > 0 ? 1u : acc0);
              else
                tc_mma_mxf4nvf4(d_tmem, pdesc + 2 * kb, qdesc + 2 * kb, idesc, sfp_col + kb * 4,
                                sfq_col + kb * C_::kSfqColsPerKb, kb > 0 ? 1u : acc0);
            }
          } else {
            const int kbv = k_blocks(ti, kt);
            for (int kb = 0; kb < kbv; ++kb) {
              if constexpr (CTA2)
                tc_mma_mxf4nvf4_2cta(d_tmem, pdesc + 2 * kb, qdesc + 2 * kb, idesc, sfp_col + kb * 4,
                                     sfq_col + kb * C_::kSfqColsPerKb, kb > 0 ? 1u : acc0);
              else
                tc_mma_mxf4nvf4(d_tmem, pdesc + 2 * kb, qdesc + 2 * kb, idesc, sfp_col + kb * 4,
                                sfq_col + kb * C_::kSfqColsPerKb, kb > 0 ? 1u : acc0);
            }
          }
          // release the stage and the TMEM scale buffer once these MMAs have read them
          if (CTA2) {
            tc_commit_2cta(empty_bar(s));
            tc_commit_2cta(sfe_bar(t));
          } else {
            tc_commit(empty_bar(s));
            tc_commit(sfe_bar(t));
          }
          if (++s == S) { s = 0; ph ^= 1; }
          if (++t == T) { t = 0; tph ^= 1; }
        }
        if (!ok) break;
        if (CTA2) tc_commit_2cta(accf_bar(acc)); else tc_commit(accf_bar(acc));
        if (++acc == A) { acc = 0; aph ^= 1; }
      }
      // wait until every tcgen05 op this thread issued has finished before TMEM is released
      if (CTA2) tc_commit_2cta(drain_bar); else tc_commit(drain_bar);
      mbar_wait_bounded(drain_bar, 0, abort_flag, prm.status, kStatusTimeoutDrain, tmo);
    }
  } else if (warp >= kFirstSfWarp) {
    {
    // -------------------------------------------------------------- scale warps
    const int grp = (warp - kFirstSfWarp) >> 2;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;  // this warp's TMEM quarter
    uint32_t tstep = 0;
    int s = 0;
    uint32_t ph = 0;
    bool ok = true;
    // Scale factors of one k-stage in registers: lane l holds row l of every atom
    // (16 bytes = 4 TMEM columns per atom), read from the stage in shared memory.
    struct SfRegs {
      uint32_t p[4 * KB];
      uint32_t q[KB * C_::kSfqColsPerKb];
    };
    auto load_stage = [&](const TileInfo& ti, int kt, int slot, int nq_atoms, SfRegs& r) {
      const int kbv = k_blocks(ti, kt);
      const uint8_t* sp = smem + slot_off(slot) + lane * 16;
      const uint8_t* sq = sp + kOffSfq;
#pragma unroll
      for (int kb = 0; kb < KB; ++kb) {
        uint4 v = make_uint4(0, 0, 0, 0);
        if (kb < kbv) v = *reinterpret_cast<const uint4*>(sp + kb * kAtomBytes);
        r.p[4 * kb + 0] = v.x; r.p[4 * kb + 1] = v.y; r.p[4 * kb + 2] = v.z; r.p[4 * kb + 3] = v.w;
      }
#pragma unroll
      for (int kb = 0; kb < KB; ++kb)
#pragma unroll
        for (int a = 0; a < C_::kSfqAtoms; ++a) {
          uint4 v = make_uint4(0, 0, 0, 0);
          if (kb < kbv && a < nq_atoms)
            v = *reinterpret_cast<const uint4*>(sq + a * KB * kAtomBytes + kb * kAtomBytes);
          const int o = kb * C_::kSfqColsPerKb + a * 4;
          r.q[o + 0] = v.x; r.q[o + 1] = v.y; r.q[o + 2] = v.z; r.q[o + 3] = v.w;
        }
    };
    auto store_stage = [&](int cs, SfRegs& r) {
      const uint32_t col = tmem_base + lane_base + C_::kSfCol0 + cs * C_::kSfCols;
      tmem_st_32x32b(col, r.p);
      tmem_st_32x32b(col + C_::kSfpCols, r.q);
    };
    // Group g serves the k-steps j with j % 2 == g.  Per step: wait until TMEM scale buffer
    // j % T is free (the MMAs of step j - T are done) and the step's scale atoms landed in
    // slot j % NS, write them, then free the slot and arrive on the buffer's sf_full (the
    // leader's, for a pair).
    // The scale atoms are loaded by the group itself: lane 0 of its first warp issues the
    // loads of the group's own steps into the group's own slots (NS is even, so slot j % NS
    // always belongs to the group of step j), NS steps ahead, and refills a slot as soon as
    // the group's four warps have read it (sf_free).  No other thread waits on these slots,
    // and no operand producer ever waits for a scale copy.
    const bool issuer = (warp & 3) == 0 && lane == 0 && !(prm.debug & 1);
    const uint64_t pol_keep = policy_evict_last();
    uint32_t sf_issued = 0, sf_par = 0;  // slots with a load issued, and that load's phase
    Cursor ic;                            // issue cursor (issuer only): global step istep
    const void* last_sf_map = nullptr;
    int istep = 0;
    auto issue_sf = [&](const Cursor& c, int slot, uint32_t par) {
      const uint32_t bar = sfd_bar(slot);
      const uint32_t dst = base + slot_off(slot);
      // two tensor loads (one per operand's scale blocks; out-of-range atoms read as zero
      // and are ignored); the grouped GEMM's per-group scale maps come from the prep kernel
      if (GROUPED && c.ti.map_sfp != last_sf_map) {
        tmap_fence_acquire(c.ti.map_sfp);
        tmap_fence_acquire(c.ti.map_sfq);
        last_sf_map = c.ti.map_sfp;
      }
      mbar_arrive_expect_tx(bar, C_::kSfSlotBytes);
      tma_load_3d(dst, c.ti.map_sfp, bar, c.kt * KB * 64, c.ti.p0 >> 7, c.ti.l, pol_keep);
      tma_load_3d(dst + kOffSfq, c.ti.map_sfq, bar, c.kt * KB * 64, c.ti.q0 >> 7, c.ti.l, pol_keep);
      sf_issued |= 1u << slot;
      sf_par = (sf_par & ~(1u << slot)) | (par << slot);
    };
    if (issuer) {  // the group's first NS / 2 steps (steps 0 .. NS-1 of its parity)
      ic.valid = seg_first<SK>(prm, total, work0, work_step, ic.sg);
      cur_load(ic);
      for (; istep < NS && ic.valid; ++istep, cur_next(ic))
        if ((istep & 1) == grp) issue_sf(ic, istep, 0u);
    }
    int sl = 0;
    uint32_t slph = 0;
    Seg sg;
    for (bool more = seg_first<SK>(prm, total, work0, work_step, sg); more && ok;
         more = seg_next<SK>(prm, total, work0, work_step, sg)) {
      TileInfo ti;
      decode_tile<GROUPED, SWAP, BN, KB, CTA2>(prm, &tm_p, &tm_q, &tm_c, &tm_sfp, &tm_sfq, sg.t, ti);
      const int nq_atoms = q_atoms(ti);
      const int kte = min(sg.kt1, ti.num_kt);
      for (int kt = sg.kt0; kt < kte && ok; ++kt, ++tstep) {
        const int cs = s;
        const uint32_t cph = ph;
        if (++s == T) { s = 0; ph ^= 1; }
        const int cslot = sl;
        const uint32_t cslph = slph;
        if (++sl == NS) { sl = 0; slph ^= 1; }
        if ((int)(tstep & 1) != grp) continue;
        int w_ok = 1;
        if (lane == 0)
          w_ok = mbar_wait_bounded(sfe_bar(cs), cph ^ 1, abort_flag, prm.status,
                                   kStatusTimeoutMma, tmo) &&
                 mbar_wait_bounded(sfd_bar(cslot), cslph, abort_flag, prm.status,
                                   kStatusTimeoutMma, tmo);
        w_ok = __shfl_sync(0xffffffffu, w_ok, 0);
        if (!w_ok) { ok = false; break; }
        tc_fence_after();
        {
          SfRegs r;
          load_stage(ti, kt, cslot, nq_atoms, r);
          store_stage(cs, r);
          tmem_st_wait();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(sfs_bar(cslot));
          arrive_leader(sff_bar(cs));
        }
        int i_ok = 1;
        if (issuer) {
          // refill the slot with step tstep + NS once the group's four warps have read it
          while (ic.valid && istep < (int)tstep + NS) {
            cur_next(ic);
            ++istep;
          }
          if (ic.valid) {
            if (mbar_wait_bounded(sfs_bar(cslot), cslph, abort_flag, prm.status,
                                  kStatusTimeoutMma, tmo))
              issue_sf(ic, cslot, cslph ^ 1u);
            else
              i_ok = 0;
          }
        }
        if (!__shfl_sync(0xffffffffu, i_ok, 0)) { ok = false; break; }
      }
    }
    if (issuer && *abort_flag) {
      // let the scale loads already issued land before the CTA exits (bounded)
      for (int i = 0; i < NS; ++i)
        if (sf_issued & (1u << i))
          mbar_wait_plain(sfd_bar(i), (sf_par >> i) & 1u, 100000000ull);
    }
    }
  } else {
    {
    // -------------------------------------------------------------- epilogue
    // Warp w owns accumulator rows 32*(w%4).. and columns [h*BN/2, (h+1)*BN/2), h = w/4.
    // It pulls its slice out of TMEM as packed fp16 (two 32-column chunks at a time),
    // releases the accumulator after the last load, and writes C with TMA stores: each
    // 16-column piece goes through one of the warp's 1 KB staging buffers in shared memory
    // (double-buffered where they fit) and leaves with one bulk tensor store.
    constexpr int kHalf = BN / 2;
    constexpr int kChunks = kHalf / 32;
    // chunks drained per store phase: the whole slice in the non-swapped order (the
    // accumulator is free before the first store), two chunks (32 registers) in the swapped
    // order, whose per-lane store addressing needs more registers (it spilled with four)
    constexpr int kPhase = (!SWAP || kChunks <= 2) ? kChunks : 2;
    int acc = 0;
    uint32_t aph = 0;
    const int quad = warp & 3;
    const int half = warp >> 2;
    const int row = quad * 32 + lane;  // TMEM lane == accumulator row
    const uint32_t epi_buf0 = base + kEpi0 + (uint32_t)(warp * C_::kEpiBufs) * 1024u;
    uint32_t epi_n = 0;  // staging buffers used so far (rotation)
    const void* last_c_map = nullptr;
    Seg sg;
    for (bool more = seg_first<SK>(prm, total, work0, work_step, sg); more;
         more = seg_next<SK>(prm, total, work0, work_step, sg)) {
      TileInfo ti;
      decode_tile<GROUPED, SWAP, BN, KB, CTA2>(prm, &tm_p, &tm_q, &tm_c, &tm_sfp, &tm_sfq, sg.t, ti);
      if (!mbar_wait_bounded(accf_bar(acc), aph, abort_flag, prm.status, kStatusTimeoutEpilogue,
                             tmo)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN + half * kHalf;
      const int q_lo = ti.q0 + half * kHalf;
      const bool fused = prm.bias || prm.act || prm.out_bf16;  // (warp-uniform)
      const int ncols = SWAP ? ti.p_rows : ti.q_rows;          // output columns N
      const int p = ti.p0 + row;
      // Store chunks c0 .. c0 + kPhase - 1 (32 columns each, packed in pk) into C itself,
      // or (n_out > 0) into every buffer of outs[].
      auto store_c = [&](__half* const Cd, const uint32_t (&pk)[kPhase][16], int c0) {
        if (p >= ti.p_rows) return;
#pragma unroll
        for (int c = 0; c < kPhase; ++c) {
          const int qc = q_lo + (c0 + c) * 32;
          if (c0 + c >= kChunks || qc >= ti.q_rows) break;
          if constexpr (!SWAP) {
            __half* dst = Cd + (long long)p * ti.ldc + qc;
            if (qc + 32 <= ti.q_rows && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
              uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
              for (int v = 0; v < 4; ++v)
                d4[v] = make_uint4(pk[c][4 * v], pk[c][4 * v + 1], pk[c][4 * v + 2], pk[c][4 * v + 3]);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (qc + j < ti.q_rows)
                  dst[j] = (j & 1) ? __high2half(*reinterpret_cast<const __half2*>(&pk[c][j >> 1]))
                                   : __low2half(*reinterpret_cast<const __half2*>(&pk[c][j >> 1]));
            }
          } else {
            // D[p=n, q=m] -> C[m, n]; lanes hold consecutive n, so each store is warp-coalesced
            __half* dst = Cd + (long long)qc * ti.ldc + p;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (qc + j < ti.q_rows)
                dst[(long long)j * ti.ldc] =
                    (j & 1) ? __high2half(*reinterpret_cast<const __half2*>(&pk[c][j >> 1]))
                            : __low2half(*reinterpret_cast<const __half2*>(&pk[c][j >> 1]));
          }
        }
      };
      // TMA store of chunks c0 .. c0 + kPhase - 1 in 16-column pieces.  Non-swapped: the
      // piece is 32 rows (lanes) x 16 columns, 32-byte rows, 32-byte swizzle.  Swapped
      // (C = D^T): 16 rows of C (the piece's q) x 32 columns (lanes), 64-byte rows, 64-byte
      // swizzle.  Rows and columns past C's edges are clipped by the TMA unit.
      const int row0 = ti.p0 + quad * 32;
      if (GROUPED && ti.c_tma && lane == 0 && ti.map_c != last_c_map) {
        tmap_fence_acquire(ti.map_c);  // written by the prep kernel through the generic proxy
        last_c_map = ti.map_c;
      }
      auto store_tma = [&](const uint32_t (&pk)[kPhase][16], int c0) {
#pragma unroll
        for (int c = 0; c < kPhase; ++c) {
          const int qc = q_lo + (c0 + c) * 32;
          if (c0 + c >= kChunks || qc >= ti.q_rows) break;  // warp-uniform
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            if (qc + hh * 16 >= ti.q_rows) break;
            const uint32_t buf = epi_buf0 + (C_::kEpiBufs == 2 ? (epi_n & 1u) * 1024u : 0u);
            ++epi_n;
            // the buffer's previous store has finished reading it
            if (lane == 0) bulk_wait_group_read<C_::kEpiBufs - 1>();
            __syncwarp();
            if constexpr (!SWAP) {
              const uint32_t rb = buf + (uint32_t)lane * 32u;
              const uint32_t sw = ((uint32_t)lane >> 2) & 1u;
              st_shared_v4(rb + (sw << 4), pk[c][hh * 8 + 0], pk[c][hh * 8 + 1], pk[c][hh * 8 + 2],
                           pk[c][hh * 8 + 3]);
              st_shared_v4(rb + ((sw ^ 1u) << 4), pk[c][hh * 8 + 4], pk[c][hh * 8 + 5],
                           pk[c][hh * 8 + 6], pk[c][hh * 8 + 7]);
            } else {
              const uint32_t col = (((uint32_t)lane & 7u) << 1);
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const uint32_t v = pk[c][hh * 8 + (j >> 1)];
                const uint32_t chunk = (((uint32_t)lane >> 3) ^ (((uint32_t)j >> 1) & 3u)) << 4;
                st_shared_u16(buf + (uint32_t)j * 64u + chunk + col,
                              (uint16_t)((j & 1) ? (v >> 16) : (v & 0xffffu)));
              }
            }
            fence_async_shared();  // make the generic-proxy writes visible to the TMA unit
            __syncwarp();
            if (lane == 0) {
              if constexpr (!SWAP) tma_store_3d(ti.map_c, buf, qc + hh * 16, row0, ti.l);
              else tma_store_3d(ti.map_c, buf, row0, qc + hh * 16, ti.l);
              bulk_commit_group();
            }
          }
        }
      };
      auto store_all = [&](const uint32_t (&pk)[kPhase][16], int c0) {
        if (prm.n_out == 0) {
          if (ti.c_tma) store_tma(pk, c0);
          else store_c(ti.C, pk, c0);
        } else {
#pragma unroll
          for (int d = 0; d < 8; ++d)
            if (d < prm.n_out) store_c(reinterpret_cast<__half*>(prm.outs[d]), pk, c0);
        }
      };
      if constexpr (SK) {
        if (sg.kt0 > 0 || sg.kt1 < ti.num_kt) {
          // ---- stream-K piece of a split tile: fp32 partials meet in the owner CTA, the
          // one holding k-step 0 (its last segment); the others (each CTA's first segment)
          // publish theirs in their slot: column group g, row r at float4 index g * 128 + r.
          float a[kHalf];
#pragma unroll
          for (int c = 0; c < kChunks; ++c)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              uint32_t r[16];
              tmem_ld_32x32b_x16(t_row + c * 32 + hh * 16, r);
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 16; ++j) a[c * 32 + hh * 16 + j] = __uint_as_float(r[j]);
            }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) arrive_leader(acce_bar(acc));
          if (++acc == A) { acc = 0; aph ^= 1; }
          const int cg0 = half * kHalf / 4;  // this warp's first column group
          float4* mine = reinterpret_cast<float4*>(prm.sk_slots) + (size_t)blockIdx.x * (BN / 4) * 128;
          if (sg.kt0 > 0) {
#pragma unroll
            for (int g = 0; g < kHalf / 4; ++g)
              __stcg(mine + (cg0 + g) * 128 + row,
                     make_float4(a[4 * g], a[4 * g + 1], a[4 * g + 2], a[4 * g + 3]));
            named_barrier_sync(1, 32 * kEpiWarps);
            if (threadIdx.x == 0) st_release_gpu(prm.sk_flags + blockIdx.x, kSkPublished);
            continue;
          }
          // later CTAs holding pieces of this tile: c in [blockIdx.x + 1, c_end)
          const int tile_end = (sg.t + 1) * prm.sk_ktn;
          int c_end = blockIdx.x + 1;
          while (c_end < (int)gridDim.x && sk_start(prm, c_end, work_step) < tile_end) ++c_end;
          if (threadIdx.x == 0) {  // wait for every piece first: one L2 round trip for all
            const uint64_t t0 = global_timer_ns();
            for (int c = blockIdx.x + 1; c < c_end; ++c) {
              while (ld_acquire_gpu(prm.sk_flags + c) != kSkPublished) {
                if (*abort_flag || global_timer_ns() - t0 > tmo) {
                  *abort_flag = 1;
                  atomicCAS(prm.status, 0, kStatusTimeoutEpilogue);
                  break;
                }
              }
              prm.sk_flags[c] = 0u;
            }
          }
          named_barrier_sync(1, 32 * kEpiWarps);
          for (int c = blockIdx.x + 1; c < c_end; ++c) {
            const float4* theirs =
                reinterpret_cast<const float4*>(prm.sk_slots) + (size_t)c * (BN / 4) * 128;
            constexpr int kRound = 8;  // float4 loads in flight per thread (register budget)
#pragma unroll
            for (int g0 = 0; g0 < kHalf / 4; g0 += kRound) {
              float4 v[kRound];
#pragma unroll
              for (int g = 0; g < kRound; ++g) v[g] = __ldcg(theirs + (cg0 + g0 + g) * 128 + row);
#pragma unroll
              for (int g = 0; g < kRound; ++g) {
                float* d = a + 4 * (g0 + g);
                d[0] += v[g].x; d[1] += v[g].y; d[2] += v[g].z; d[3] += v[g].w;
              }
            }
          }
          static_assert(!SK || kPhase == kChunks, "stream-K tiles are stored in one phase");
          uint32_t pk[kPhase][16];
#pragma unroll
          for (int c = 0; c < kPhase; ++c)
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int n0 = SWAP ? ti.p0 + row : q_lo + c * 32 + 2 * j;
              const int n1 = SWAP ? n0 : n0 + 1;
              pk[c][j] = epi_pack(prm, epi_post(prm, a[c * 32 + 2 * j], n0, ncols),
                                  epi_post(prm, a[c * 32 + 2 * j + 1], n1, ncols));
            }
          store_all(pk, 0);
          continue;
        }
      }
      if constexpr (F32) {
        {
          // fp32 C: the 32-bit values would double the packed tile's registers, so each
          // 16-column piece is stored straight from its TMEM load and the accumulator is
          // released after the last store.
          float* const Cf = reinterpret_cast<float*>(prm.C) + (long long)ti.l * prm.c_batch;
          const int p = ti.p0 + row;
#pragma unroll 1
          for (int c = 0; c < kChunks; ++c) {
            if (q_lo + c * 32 >= ti.q_rows) break;  // warp-uniform
#pragma unroll 1
            for (int hh = 0; hh < 2; ++hh) {
              uint32_t r[16];
              tmem_ld_32x32b_x16(t_row + c * 32 + hh * 16, r);
              tmem_ld_wait();
              const int qb = q_lo + c * 32 + hh * 16;
              float v[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) v[j] = epi_post(prm, __uint_as_float(r[j]), SWAP ? p : qb + j, ncols);
              if (p >= ti.p_rows) continue;
              if constexpr (!SWAP) {
                float* dst = Cf + (long long)p * ti.ldc + qb;
                if (qb + 16 <= ti.q_rows && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
                  for (int w = 0; w < 4; ++w)
                    reinterpret_cast<float4*>(dst)[w] = make_float4(v[4 * w], v[4 * w + 1], v[4 * w + 2], v[4 * w + 3]);
                } else {
#pragma unroll
                  for (int j = 0; j < 16; ++j)
                    if (qb + j < ti.q_rows) dst[j] = v[j];
                }
              } else {
                // D[p=n, q=m] -> C[m, n]: lanes hold consecutive n (coalesced per j)
                float* dst = Cf + (long long)qb * ti.ldc + p;
#pragma unroll
                for (int j = 0; j < 16; ++j)
                  if (qb + j < ti.q_rows) dst[(long long)j * ti.ldc] = v[j];
              }
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) arrive_leader(acce_bar(acc));
          if (++acc == A) { acc = 0; aph ^= 1; }
          continue;
        }
      }
      // Drain kPhase chunks of 32 columns into registers as packed fp16/bf16, store them,
      // then the next kPhase.  The accumulator is
      // released right after its last TMEM load; the MMAs of the next tile wait at most
      // for the issue of the earlier phases' stores (fire-and-forget).
#pragma unroll
      for (int c0 = 0; c0 < kChunks; c0 += kPhase) {
        uint32_t pk[kPhase][16];
#pragma unroll
        for (int cc = 0; cc < kPhase; ++cc) {
          const int c = c0 + cc;
          if (c < kChunks && q_lo + c * 32 < ti.q_rows) {  // warp-uniform (BN = 192: 3 chunks)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              uint32_t r[16];
              tmem_ld_32x32b_x16(t_row + c * 32 + hh * 16, r);
              tmem_ld_wait();
              if (!fused) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  __half2 h = __floats2half2_rn(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
                  pk[cc][hh * 8 + j] = *reinterpret_cast<uint32_t*>(&h);
                }
              } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  const int n0 = SWAP ? ti.p0 + row : q_lo + c * 32 + hh * 16 + 2 * j;
                  const int n1 = SWAP ? n0 : n0 + 1;
                  pk[cc][hh * 8 + j] = epi_pack(prm, epi_post(prm, __uint_as_float(r[2 * j]), n0, ncols),
                                                epi_post(prm, __uint_as_float(r[2 * j + 1]), n1, ncols));
                }
              }
            }
          }
        }
        if (c0 + kPhase >= kChunks) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) arrive_leader(acce_bar(acc));
          if (++acc == A) { acc = 0; aph ^= 1; }
        }
        store_all(pk, c0);
      }
    }
    // the CTA's shared memory must outlive the TMA stores that read it
    if (lane == 0) bulk_wait_group_all();
    }
  }

  tc_fence_before();
  __syncthreads();
  // Pair: neither CTA leaves (or frees TMEM) while the leader's MMAs may still read the
  // peer's shared memory or the peer still arrives on the leader's barriers.
  if (CTA2) cluster_sync();
  if (warp == kMmaWarp) {
    __syncwarp();
    tc_fence_after();
    if (CTA2) tmem_dealloc_2cta(tmem_base, C_::kTmemCols);
    else tmem_dealloc(tmem_base, C_::kTmemCols);
  }
}

#pragma nv_diagnostic pop

}  // namespace nvfp4
