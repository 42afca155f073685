// NVFP4 block-scaled GEMM kernels for sm_100a (B200).
//
// One persistent, warp-specialised kernel body serves both the dense GEMM
// (kernels/gemm/submission.py:51-583 in the reference) and the grouped GEMM
// (kernels/group_gemm/submission.py:55-703).  It computes
//
//     D[p, q] = sum_k  e2m1(P[p, k]) * sfP[p, k/16]  *  e2m1(Q[q, k]) * sfQ[q, k/16]
//
// in fp32 in tensor memory and stores fp16.  P is the operand that feeds the
// 128-row MMA M side, Q the operand that feeds the MMA N side (BN rows).  For
// the ordinary layout P = A (M rows) and Q = B (N rows) and C[m, n] = D[m, n];
// for "swap" P = B and Q = A and C[m, n] = D[n, m], which lets a skinny M
// (decode-like shapes, small MoE groups) sit on the flexible N side of the MMA.
//
// Roles (192 threads):
//   warps 0-3  epilogue: TMEM -> registers -> fp16 -> global (warp w owns TMEM lanes 32w..32w+31)
//   warp 4     producer: TMA tiles of P and Q (128-byte swizzle) + bulk copies of the
//              scale-factor atoms into an mbarrier ring of STAGES stages
//   warp 5     TMEM owner and MMA issuer: tcgen05.cp scale atoms into TMEM, then
//              tcgen05.mma kind::mxf4nvf4 (K = 64 per instruction, 4 per stage)
//
// Scale factors arrive in the reference's pre-permuted layout
// (kernels/gemm/reference.py:113-150): per 128-row block and per 64-wide K block
// one 512-byte atom whose byte (r % 32) * 16 + (r / 32) * 4 + j holds row r,
// K-vector j.  The four atoms of one 256-wide K stage are contiguous (2 KiB),
// so they are fetched with one plain bulk copy, and tcgen05.cp 32x128b.warpx4
// puts an atom into four TMEM columns in exactly the order the MMA reads it
// (column c, lane l <-> row 32c + l).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>
#include "ptx_sm100.cuh"

namespace nvfp4 {

constexpr int kBM = 128;            // MMA M (rows of P per tile)
constexpr int kBKBytes = 128;       // bytes of K per stage (256 fp4 values)
constexpr int kBK = 256;            // K elements per stage
constexpr int kMmaK = 64;           // K per tcgen05.mma
constexpr int kAtomBytes = 512;     // one scale-factor atom: 128 rows x 4 K-vectors
constexpr int kNumThreads = 192;
constexpr int kProducerWarp = 4;
constexpr int kMmaWarp = 5;
constexpr int kSmemBudget = 232448 - 2048;  // dynamic smem per CTA minus alignment/barriers

template <int BN>
struct Cfg {
  static_assert(BN == 32 || BN == 64 || BN == 128 || BN == 192 || BN == 256,
                "BN must be 32, 64, 128, 192 or 256 (tiles start on 32-row boundaries of a scale block)");
  static constexpr int kPBytes = kBM * kBKBytes;
  static constexpr int kQBytes = BN * kBKBytes;
  // 128-row scale blocks a Q tile can touch (a tile may start at row 64 of a block).
  static constexpr int kSfqAtoms = (BN <= 128) ? 1 : 2;
  static constexpr int kSfpBytes = 4 * kAtomBytes;
  static constexpr int kSfqBytes = kSfqAtoms * 4 * kAtomBytes;
  static constexpr int kStageBytes = kPBytes + kQBytes + kSfpBytes + kSfqBytes;
  static constexpr int kStagesRaw = kSmemBudget / kStageBytes;
  static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
  static constexpr int kSfqColsPerKb = 4 * kSfqAtoms;
  static constexpr int kSfCols = 4 * 4 + 4 * kSfqColsPerKb;
  static constexpr int kAccStages = (2 * BN + kSfCols <= 512) ? 2 : 1;
  static constexpr int kColsNeeded = kAccStages * BN + kSfCols;
  static constexpr int kTmemCols = kColsNeeded <= 32 ? 32 : kColsNeeded <= 64 ? 64
                                 : kColsNeeded <= 128 ? 128 : kColsNeeded <= 256 ? 256 : 512;
  static constexpr int kSfpCol = kAccStages * BN;
  static constexpr int kSfqCol = kSfpCol + 16;
  // barriers: full[S], empty[S], acc_full[A], acc_empty[A], drain; then tmem ptr + abort flag
  static constexpr int kBarrierBytes = 8 * (2 * kStages + 2 * kAccStages + 1) + 16;
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kBarrierBytes;
  static_assert(kStages >= 2, "not enough shared memory for two stages");
  static_assert(kColsNeeded <= 512, "TMEM budget exceeded");
};

// Everything the kernel needs; tensor maps for the dense case are separate
// __grid_constant__ parameters.
struct GemmParams {
  // dense problem (ignored when grouped)
  int p_rows, q_rows, K, L;
  const uint8_t* sf_p;          // permuted scale factors of P
  const uint8_t* sf_q;          // permuted scale factors of Q
  long long sf_p_batch;         // bytes between batches
  long long sf_q_batch;
  __half* C;
  long long ldc;                // elements between rows of C
  long long c_batch;            // elements between batches of C
  int tiles_p, tiles_q, total_tiles;
  int q_fastest;                // raster order: 1 = walk Q tiles first
  // grouped problem
  int G;
  const int* sizes;             // G x 4: m, n, k, l
  const unsigned long long* abc;  // G x 3: a, b, c
  const unsigned long long* sfs;  // G x 2: sfa (permuted), sfb (permuted)
  const CUtensorMap* maps;      // G x 2: [P map = B_g, Q map = A_g]
  const int* tile_prefix;       // G + 1 running tile counts
  // control
  int* status;
  unsigned long long timeout_ns;
  int debug_skip_producer;      // test hook: producer issues nothing, waits must time out
};

// Per-tile view shared by all roles.
struct TileInfo {
  int p0, q0, l;
  int p_rows, q_rows, K;
  const void* map_p;
  const void* map_q;
  const uint8_t* sf_p;   // batch-adjusted base
  const uint8_t* sf_q;
  __half* C;             // batch-adjusted base
  long long ldc;
  int rk;                // 64-wide K blocks (atoms per 128-row block)
  int num_kt;            // 256-wide K stages
};

template <bool GROUPED, bool SWAP, int BN>
__device__ __forceinline__ bool decode_tile(const GemmParams& prm, const CUtensorMap* tm_p,
                                            const CUtensorMap* tm_q, int t, TileInfo& ti) {
  if constexpr (!GROUPED) {
    const int per_batch = prm.tiles_p * prm.tiles_q;
    const int l = t / per_batch;
    const int r = t - l * per_batch;
    int pb, qb;
    if (prm.q_fastest) { qb = r % prm.tiles_q; pb = r / prm.tiles_q; }
    else               { pb = r % prm.tiles_p; qb = r / prm.tiles_p; }
    ti.p0 = pb * kBM;
    ti.q0 = qb * BN;
    ti.l = l;
    ti.p_rows = prm.p_rows;
    ti.q_rows = prm.q_rows;
    ti.K = prm.K;
    ti.map_p = tm_p;
    ti.map_q = tm_q;
    ti.sf_p = prm.sf_p + (long long)l * prm.sf_p_batch;
    ti.sf_q = prm.sf_q + (long long)l * prm.sf_q_batch;
    ti.C = prm.C + (long long)l * prm.c_batch;
    ti.ldc = prm.ldc;
    ti.rk = (prm.K + 63) / 64;
    ti.num_kt = (prm.K + kBK - 1) / kBK;
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
    // swap layout: P = B_g (n rows), Q = A_g (m rows); walk Q (token) tiles first
    const int tq = (m + BN - 1) / BN;
    const int qb = r % tq;
    const int pb = r / tq;
    ti.p0 = pb * kBM;
    ti.q0 = qb * BN;
    ti.l = 0;
    ti.p_rows = n;
    ti.q_rows = m;
    ti.K = k;
    ti.map_p = prm.maps + 2 * g;
    ti.map_q = prm.maps + 2 * g + 1;
    ti.sf_p = reinterpret_cast<const uint8_t*>(__ldg(prm.sfs + 2 * g + 1));
    ti.sf_q = reinterpret_cast<const uint8_t*>(__ldg(prm.sfs + 2 * g + 0));
    ti.C = reinterpret_cast<__half*>(__ldg(prm.abc + 3 * g + 2));
    ti.ldc = n;
    ti.rk = (k + 63) / 64;
    ti.num_kt = (k + kBK - 1) / kBK;
    return true;
  }
}

template <bool GROUPED, bool SWAP, int BN>
__global__ void __launch_bounds__(kNumThreads, 1)
nvfp4_gemm_kernel(const __grid_constant__ CUtensorMap tm_p, const __grid_constant__ CUtensorMap tm_q,
                  const GemmParams prm) {
  using C_ = Cfg<BN>;
  constexpr int S = C_::kStages;
  constexpr int A = C_::kAccStages;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);

  // stage s: [P | Q | SFP | SFQ]
  auto stage_p = [&](int s) { return base + s * C_::kStageBytes; };
  auto stage_q = [&](int s) { return base + s * C_::kStageBytes + C_::kPBytes; };
  auto stage_sfp = [&](int s) { return base + s * C_::kStageBytes + C_::kPBytes + C_::kQBytes; };
  auto stage_sfq = [&](int s) {
    return base + s * C_::kStageBytes + C_::kPBytes + C_::kQBytes + C_::kSfpBytes;
  };
  const uint32_t bar_base = base + S * C_::kStageBytes;
  auto full_bar = [&](int s) { return bar_base + 8 * s; };
  auto empty_bar = [&](int s) { return bar_base + 8 * (S + s); };
  auto accf_bar = [&](int a) { return bar_base + 8 * (2 * S + a); };
  auto acce_bar = [&](int a) { return bar_base + 8 * (2 * S + A + a); };
  const uint32_t drain_bar = bar_base + 8 * (2 * S + 2 * A);
  uint8_t* bar_ptr = smem + S * C_::kStageBytes;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(bar_ptr + 8 * (2 * S + 2 * A + 1));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bar_ptr + 8 * (2 * S + 2 * A + 1) + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < A; ++a) {
      mbar_init(accf_bar(a), 1);
      mbar_init(acce_bar(a), 128);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
    fence_async_shared();
  }
  if (warp == kProducerWarp && lane == 0 && !GROUPED) {
    prefetch_tmap(&tm_p);
    prefetch_tmap(&tm_q);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(const_cast<uint32_t*>(tmem_slot)), C_::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int total = GROUPED ? __ldg(prm.tile_prefix + prm.G) : prm.total_tiles;
  const uint64_t tmo = prm.timeout_ns;

  if (warp == kProducerWarp) {
    if (lane == 0 && !prm.debug_skip_producer) {
      // ------------------------------------------------------------ producer
      const uint64_t pol_stream = policy_evict_first();
      const uint64_t pol_keep = policy_evict_last();
      int s = 0;
      uint32_t ph = 0;
      const void* last_map = nullptr;
      bool ok = true;
      uint32_t issued_mask = 0, issued_par = 0;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        TileInfo ti;
        decode_tile<GROUPED, SWAP, BN>(prm, &tm_p, &tm_q, t, ti);
        if (GROUPED && ti.map_p != last_map) {
          tmap_fence_acquire(ti.map_p);
          tmap_fence_acquire(ti.map_q);
          last_map = ti.map_p;
        }
        const int pblk = ti.p0 >> 7;
        const int qblk = ti.q0 >> 7;
        const int rq = (ti.q_rows + 127) >> 7;
        int nq_atoms = ((ti.q0 & 127) + BN + 127) >> 7;
        if (nq_atoms > C_::kSfqAtoms) nq_atoms = C_::kSfqAtoms;
        if (qblk + nq_atoms > rq) nq_atoms = rq - qblk;
        // P (the operand re-read by several tiles in flight) stays in L2 longer
        const uint64_t pol_p = pol_keep;
        const uint64_t pol_q = pol_stream;
        (void)pol_q;
        for (int kt = 0; kt < ti.num_kt; ++kt) {
          if (!mbar_wait_bounded(empty_bar(s), ph ^ 1, abort_flag, prm.status,
                                 kStatusTimeoutProducer, tmo)) { ok = false; break; }
          int kbv = ti.rk - kt * 4;
          if (kbv > 4) kbv = 4;
          const uint32_t sf_bytes = kbv * kAtomBytes;
          const uint32_t bytes = C_::kPBytes + C_::kQBytes + sf_bytes * (1 + nq_atoms);
          mbar_arrive_expect_tx(full_bar(s), bytes);
          tma_load_3d(stage_p(s), ti.map_p, full_bar(s), kt * kBKBytes, ti.p0, ti.l, pol_p);
          tma_load_3d(stage_q(s), ti.map_q, full_bar(s), kt * kBKBytes, ti.q0, ti.l, pol_keep);
          bulk_load(stage_sfp(s), ti.sf_p + ((long long)pblk * ti.rk + kt * 4) * kAtomBytes,
                    sf_bytes, full_bar(s), pol_keep);
          for (int a = 0; a < nq_atoms; ++a)
            bulk_load(stage_sfq(s) + a * 4 * kAtomBytes,
                      ti.sf_q + ((long long)(qblk + a) * ti.rk + kt * 4) * kAtomBytes, sf_bytes,
                      full_bar(s), pol_keep);
          issued_mask |= 1u << s;
          issued_par = (issued_par & ~(1u << s)) | (ph << s);
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
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      int s = 0;
      uint32_t ph = 0;
      int acc = 0;
      uint32_t aph = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        TileInfo ti;
        decode_tile<GROUPED, SWAP, BN>(prm, &tm_p, &tm_q, t, ti);
        int n_mma = ti.q_rows - ti.q0;
        if (n_mma > BN) n_mma = BN;
        n_mma = (n_mma + 15) & ~15;
        const uint32_t idesc = make_idesc_mxf4nvf4(kBM, n_mma);
        const uint32_t d_tmem = tmem_base + acc * BN;
        const uint32_t sfq_shift = (ti.q0 & 127) >> 5;
        const int rq = (ti.q_rows + 127) >> 7;
        int nq_atoms = ((ti.q0 & 127) + BN + 127) >> 7;
        if (nq_atoms > C_::kSfqAtoms) nq_atoms = C_::kSfqAtoms;
        if ((ti.q0 >> 7) + nq_atoms > rq) nq_atoms = rq - (ti.q0 >> 7);
        if (!mbar_wait_bounded(acce_bar(acc), aph ^ 1, abort_flag, prm.status, kStatusTimeoutMma,
                               tmo)) { ok = false; break; }
        tc_fence_after();
        for (int kt = 0; kt < ti.num_kt; ++kt) {
          if (!mbar_wait_bounded(full_bar(s), ph, abort_flag, prm.status, kStatusTimeoutMma, tmo)) {
            ok = false;
            break;
          }
          tc_fence_after();
          int kbv = ti.rk - kt * 4;
          if (kbv > 4) kbv = 4;
          for (int kb = 0; kb < kbv; ++kb) {
            tc_cp_32x128b_warpx4(tmem_base + C_::kSfpCol + kb * 4,
                                 make_smem_desc(stage_sfp(s) + kb * kAtomBytes, 0, 128, 0));
            for (int a = 0; a < nq_atoms; ++a)
              tc_cp_32x128b_warpx4(
                  tmem_base + C_::kSfqCol + kb * C_::kSfqColsPerKb + a * 4,
                  make_smem_desc(stage_sfq(s) + a * 4 * kAtomBytes + kb * kAtomBytes, 0, 128, 0));
          }
          const uint64_t pdesc = make_smem_desc(stage_p(s), 0, 1024, 2);
          const uint64_t qdesc = make_smem_desc(stage_q(s), 0, 1024, 2);
          for (int kb = 0; kb < kbv; ++kb) {
            // advance 32 bytes (64 fp4) along K inside the 128-byte swizzled row
            tc_mma_mxf4nvf4(d_tmem, pdesc + 2 * kb, qdesc + 2 * kb, idesc,
                            tmem_base + C_::kSfpCol + kb * 4,
                            tmem_base + C_::kSfqCol + kb * C_::kSfqColsPerKb + sfq_shift,
                            (kt > 0 || kb > 0) ? 1u : 0u);
          }
          tc_commit(empty_bar(s));
          if (++s == S) { s = 0; ph ^= 1; }
        }
        if (!ok) break;
        tc_commit(accf_bar(acc));
        if (++acc == A) { acc = 0; aph ^= 1; }
      }
      // wait until every tcgen05 op this thread issued has finished before TMEM is released
      tc_commit(drain_bar);
      mbar_wait_bounded(drain_bar, 0, abort_flag, prm.status, kStatusTimeoutDrain, tmo);
    }
  } else {
    // -------------------------------------------------------------- epilogue
    int acc = 0;
    uint32_t aph = 0;
    const int row = warp * 32 + lane;  // TMEM lane == accumulator row
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      TileInfo ti;
      decode_tile<GROUPED, SWAP, BN>(prm, &tm_p, &tm_q, t, ti);
      if (!mbar_wait_bounded(accf_bar(acc), aph, abort_flag, prm.status, kStatusTimeoutEpilogue,
                             tmo)) break;
      tc_fence_after();
      const int p = ti.p0 + row;
      const bool p_ok = p < ti.p_rows;
      const uint32_t t_row = tmem_base + ((uint32_t)(warp * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        const int qc = ti.q0 + c * 32;
        if (qc >= ti.q_rows) break;  // warp-uniform
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + c * 32, r);
        tmem_ld_wait();
        if (!p_ok) continue;
        if constexpr (!SWAP) {
          __half* dst = ti.C + (long long)p * ti.ldc + qc;
          const bool full = (qc + 32 <= ti.q_rows) &&
                            ((reinterpret_cast<uintptr_t>(dst) & 15) == 0);
          if (full) {
            uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint4 w;
              __half2 h0 = __floats2half2_rn(__uint_as_float(r[8 * v + 0]), __uint_as_float(r[8 * v + 1]));
              __half2 h1 = __floats2half2_rn(__uint_as_float(r[8 * v + 2]), __uint_as_float(r[8 * v + 3]));
              __half2 h2 = __floats2half2_rn(__uint_as_float(r[8 * v + 4]), __uint_as_float(r[8 * v + 5]));
              __half2 h3 = __floats2half2_rn(__uint_as_float(r[8 * v + 6]), __uint_as_float(r[8 * v + 7]));
              w.x = *reinterpret_cast<uint32_t*>(&h0);
              w.y = *reinterpret_cast<uint32_t*>(&h1);
              w.z = *reinterpret_cast<uint32_t*>(&h2);
              w.w = *reinterpret_cast<uint32_t*>(&h3);
              d4[v] = w;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (qc + j < ti.q_rows) dst[j] = __float2half_rn(__uint_as_float(r[j]));
          }
        } else {
          // D[p=n, q=m] -> C[m, n]; lanes hold consecutive n, so each store is warp-coalesced
          __half* dst = ti.C + (long long)qc * ti.ldc + p;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (qc + j < ti.q_rows) dst[(long long)j * ti.ldc] = __float2half_rn(__uint_as_float(r[j]));
        }
      }
      tc_fence_before();
      mbar_arrive(acce_bar(acc));
      if (++acc == A) { acc = 0; aph ^= 1; }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, C_::kTmemCols);
  }
}

}  // namespace nvfp4
