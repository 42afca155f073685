/*
 * nvfp4_b200.h - C ABI of the B200-native NVFP4 block-scaled GEMM library.
 *
 * Data formats (identical to the reference's input tuples):
 *   a, b      : e2m1 codes, two per byte (element 2i in the low nibble),
 *               K-major; a is (L, M, K/2) bytes, b is (L, N, K/2) bytes.
 *               (kernels/gemm/reference.py:86-93, task.py:4)
 *   sf*_perm  : e4m3 scale factors, one per 16 elements along K, in the
 *               pre-permuted 128x4 "blocked" layout: storage order
 *               (L, ceil(MN/128), ceil(K/64), 32, 4, 4) bytes; row r, K-vector j
 *               of one 128-row block sits at byte (r%32)*16 + (r/32)*4 + j%4 of
 *               atom (j/4).  (kernels/gemm/reference.py:113-150)
 *   c         : fp16, (L, M, N) row-major, written in place (no beta).
 * Computation: C = fp16( sum_k e2m1(A)*sfA * e2m1(B)*sfB ), fp32 accumulation.
 *
 * Every entry point launches on the given CUDA stream (cudaStream_t passed
 * as void*, NULL = legacy default stream) and never synchronises it.  Return
 * value 0 = launched; otherwise an NVFP4_ERR_* code, with a message from
 * nvfp4_last_error().  Device-side failures (a pipeline wait that ran out,
 * a bad group entry) are recorded in a per-device status word (see
 * nvfp4_status_get()), or in the caller's own word (nvfp4_options.dev_status).
 */
#ifndef NVFP4_B200_H
#define NVFP4_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NVFP4_ABI_VERSION 2

#define NVFP4_OK 0
#define NVFP4_ERR_INVALID_ARG 1   /* null pointer, non-positive size, bad group table */
#define NVFP4_ERR_ALIGNMENT 2     /* a/b/scales not 16-byte aligned, c not 2-byte aligned */
#define NVFP4_ERR_UNSUPPORTED 3   /* k not a multiple of 64, wrong GPU, too many groups */
#define NVFP4_ERR_CUDA 4          /* a CUDA runtime call failed */
#define NVFP4_ERR_DRIVER 5        /* tensor-map encoding through the driver failed */
#define NVFP4_ERR_WORKSPACE 6     /* workspace missing or too small */

/* Device status word values (nvfp4_status_get). */
#define NVFP4_STATUS_OK 0
#define NVFP4_STATUS_TIMEOUT_PRODUCER 1
#define NVFP4_STATUS_TIMEOUT_MMA 2
#define NVFP4_STATUS_TIMEOUT_EPILOGUE 3
#define NVFP4_STATUS_TIMEOUT_DRAIN 4
#define NVFP4_STATUS_BAD_GROUP 5

/* Tuning / test knobs; zero-initialise and set what you need. */
typedef struct nvfp4_options {
  int operand_order;              /* 0 = auto; 1 = A feeds the 128-row MMA side;
                                     2 = B feeds it ("swap", for skinny M).  Grouped GEMM:
                                     0 / 2 = B_g on the 128-row side, tokens on the N side;
                                     1 = tokens (A_g) on the 128-row side, tile_n 128 or 256
                                     rows of B_g on the N side (256 with cta_pair = 2) */
  int tile_n;                     /* 0 = library default; else 64, 128 or 256 (grouped: also 192) */
  int max_ctas;                   /* 0 = one CTA per SM */
  unsigned long long timeout_ns;  /* 0 = library default (2 s per pipeline wait) */
  int debug;                      /* test bit, 0 in normal use: 1 = issue no loads, so every
                                     pipeline wait runs out (the timeout path's test) */
  int* dev_status;                /* NULL = record device-side errors in the per-device status
                                     word (nvfp4_status_get); else a device int of the caller's
                                     that this call's kernels record their first error into
                                     (atomicCAS from 0: the caller clears it before the call) */
  int stage_k;                    /* 0 = auto; 128 or 256 K elements per pipeline stage */
  int cta_pair;                   /* 0 = auto (dense: pairs for M >= 256 with N >= 2048), 1 = off,
                                     2 = 256-row tiles on a CTA pair (cta_group::2; grouped:
                                     tile_n 128 or 256) */
  int stream_k;                   /* dense: 0 / 1 = off, 2 = on (k-steps split evenly over all SMs).  Stream-K
                                     keeps a per-stream workspace (flags + fp32 partials, ~16 MiB),
                                     allocated by the first stream-K call on that stream (outside
                                     any capture of it); its flags are cleared by a memset on the
                                     stream before every stream-K launch */
  /* Fused epilogue, dense GEMM only (the grouped entry points reject it):
   *   C[m, n] = act(acc[m, n] + bias[n]), rounded to the output type. */
  const float* bias;              /* NULL, or N fp32 values (device), the same for every batch */
  int activation;                 /* 0 = none, 1 = relu, 2 = gelu (erf form) */
  int out_dtype;                  /* 0 = fp16, 1 = bf16, 2 = fp32 (c holds that type; fp32:
                                     dense plain schedule, not with stream_k) */
} nvfp4_options;

/* Human-readable message for the last error returned on this thread. */
const char* nvfp4_last_error(void);
int nvfp4_abi_version(void);

/* Per-wait timeout used by kernels launched afterwards (0 restores 2 s). */
int nvfp4_set_timeout_ns(unsigned long long ns);

/* Synchronous read / reset of the current device's status word. */
int nvfp4_status_get(int* out);
int nvfp4_status_reset(void);

/*
 * Dense NVFP4 GEMM, C[l] = A[l] * B[l]^T.
 * Replaces custom_kernel() of kernels/gemm/submission.py:772-794 (which reads
 * a, b, sfa_permuted, sfb_permuted, c and writes c in place) and its launch
 * path my_kernel(), kernels/gemm/submission.py:586-746.
 * Requirements: m, n, l >= 1; k >= 64 and k % 64 == 0.
 */
int nvfp4_gemm(const void* a, const void* b, const void* sfa_perm, const void* sfb_perm, void* c,
               int m, int n, int k, int l, void* stream);

/* Same as nvfp4_gemm with tuning / test options (opt may be NULL). */
int nvfp4_gemm_ex(const void* a, const void* b, const void* sfa_perm, const void* sfb_perm, void* c,
                  int m, int n, int k, int l, void* stream, const nvfp4_options* opt);

/*
 * Grouped NVFP4 GEMM: for every group g, C_g = A_g * B_g^T (l must be 1).
 * Replaces custom_kernel() of kernels/group_gemm/submission.py:962-1087 and its
 * device tables (problem sizes G x 4 int32, a/b/c pointers G x 3 int64,
 * sfa/sfb permuted-scale pointers G x 2 int64: submission.py:993-1013).
 * All three tables are DEVICE pointers, so a router kernel can fill them
 * without a host round trip; groups with m == 0 or n == 0 are skipped.
 * workspace: device memory of nvfp4_grouped_gemm_workspace_size(G) bytes,
 * 256-byte aligned, not shared with a call in flight on another stream.
 * Requirements per group: k % 64 == 0, k >= 64, a/b/sf 16-byte aligned.
 * A group that violates them is skipped and NVFP4_STATUS_BAD_GROUP is
 * recorded in the status word.  1 <= G <= 1024.
 */
size_t nvfp4_grouped_gemm_workspace_size(int G);

int nvfp4_grouped_gemm(const int32_t* sizes_dev, const uint64_t* abc_ptrs_dev,
                       const uint64_t* sf_ptrs_dev, int G, void* workspace, size_t workspace_bytes,
                       void* stream);

/* Same with tuning / test options (tile_n = 64, 128, 192 or 256 token rows per tile). */
int nvfp4_grouped_gemm_ex(const int32_t* sizes_dev, const uint64_t* abc_ptrs_dev,
                          const uint64_t* sf_ptrs_dev, int G, void* workspace,
                          size_t workspace_bytes, void* stream, const nvfp4_options* opt);

/*
 * Dense GEMM writing C into several buffers at once (L = 1): outs[0 .. n_out), n_out <= 8,
 * each already offset to this GEMM's first column, row stride ldc elements.  With the
 * buffers of other GPUs (opened below) this is the N-sharded GEMM fused with the all-gather
 * of C (configs[4] of the benchmark): every rank computes C[:, its columns] and its epilogue
 * stores the tiles into every rank's full C over NVLink.  The reference has no multi-GPU
 * path; the unfused form is its GEMM (kernels/gemm/submission.py:772-794) followed by an
 * NCCL all-gather.  Callers order the peers' reads after this kernel (e.g. a barrier).
 */
int nvfp4_gemm_multi(const void* a, const void* b, const void* sfa_perm, const void* sfb_perm,
                     const void* const* outs, int n_out, long long ldc, int m, int n, int k,
                     void* stream);

/* CUDA IPC for the buffers above: export a device pointer (handle of its allocation plus
 * the pointer's offset in it), open a peer's handle (returns the allocation's base; add the
 * offset), close it again.  nvfp4_ipc_handle_size() bytes per handle. */
int nvfp4_ipc_handle_size(void);
int nvfp4_ipc_get_handle(const void* dev_ptr, void* handle_out, unsigned long long* offset_out);
int nvfp4_ipc_open_handle(const void* handle, void** dev_ptr_out);
int nvfp4_ipc_close(void* dev_ptr);

/*
 * Quantise x to NVFP4 on the GPU: the inputs the GEMMs take, computed from real values.
 * Replaces the host-side generation steps of the reference (kernels/gemm/reference.py:86-150:
 * per-16-element amax / 6 -> e4m3 scale, nearest e2m1 code, to_blocked scale permutation),
 * which the reference runs with torch ops before the timed GEMM.
 *   x        : (l, rows, k) contiguous, dtype NVFP4_DTYPE_F32 / _F16 / _BF16
 *   codes    : (l, rows, k/2) bytes, element 2i in the low nibble
 *   sf_perm  : (l, ceil(rows/128), k/64, 512) bytes, the permuted layout (padding rows 0)
 *   sf_plain : NULL, or (l, rows, k/16) bytes
 * Rounding: scale = e4m3(amax / 6) to nearest even (out of range -> NaN), code = nearest
 * e2m1 of |x| / scale clamped to 6, ties to the even code.  Requirements: k % 64 == 0;
 * x, codes, sf_perm 16-byte aligned.
 */
#define NVFP4_DTYPE_F32 0
#define NVFP4_DTYPE_F16 1
#define NVFP4_DTYPE_BF16 2
int nvfp4_quantize(const void* x, int dtype, int rows, int k, int l, void* codes, void* sf_perm,
                   void* sf_plain, void* stream);

/*
 * Grouped NVFP4 GEMM that allocates nothing.  No counterpart in the reference;
 * it is for callers that must not allocate device memory at call time, such as
 * code running inside a pre-planned memory pool or a host runtime that owns
 * every allocation itself, and so cannot provide the workspace that
 * nvfp4_grouped_gemm wants.  Same tables, same results as nvfp4_grouped_gemm
 * with default options.
 * Limit: 1 <= G <= 256 (larger G is rejected with NVFP4_ERR_UNSUPPORTED).
 * The scratch (about 161 KiB for the per-group tensor maps and tile schedule) is
 * a fixed device array inside the library; each GPU that loads the library
 * holds it until the process exits.  The first call on a device looks up that
 * array's address (with that device current); make that first call before any
 * stream capture.  All calls on a device share the one array, so two calls
 * that may run at the same time on the GPU (different streams, no ordering
 * between them) race and give wrong results; calls on one stream are fine.
 */
int nvfp4_grouped_gemm_noalloc(const int32_t* sizes_dev, const uint64_t* abc_ptrs_dev,
                               const uint64_t* sf_ptrs_dev, int G, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NVFP4_B200_H */
