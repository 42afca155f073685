/*
 * A plain C caller of the library's C ABI (include/nvfp4_b200.h): no Python, no torch.
 * It builds NVFP4 operands on the host, uploads them with the CUDA runtime, calls
 * nvfp4_gemm / nvfp4_gemm_ex / nvfp4_grouped_gemm, and checks every output element against
 * a double-precision restatement of the reference's math (kernels/gemm/reference.py:27-53:
 * C = fp16(sum_k e2m1(A) * e4m3(sfA) * e2m1(B) * e4m3(sfB))) at the reference checker's
 * tolerance, rtol = atol = 1e-3 (kernels/gemm/reference.py:161).  It also checks the
 * argument errors.  Exit status 0 = all checks passed.
 *
 * Build: gcc -std=c99 -O2 nvfp4_c_check.c -I<repo>/include -I<cuda>/include
 *        -L<repo>/nvfp4_hackathon_b200 -lnvfp4_b200 -L<cuda>/lib64 -lcudart -lm
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "nvfp4_b200.h"

static uint64_t rng_state = 0x9E3779B97F4A7C15ull;
static uint32_t rng(void) {  /* xorshift64* */
  rng_state ^= rng_state >> 12;
  rng_state ^= rng_state << 25;
  rng_state ^= rng_state >> 27;
  return (uint32_t)((rng_state * 2685821657736338717ull) >> 32);
}

static double e2m1(int code) {
  static const double mag[8] = {0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0};
  return (code & 8) ? -mag[code & 7] : mag[code & 7];
}

static double e4m3(uint8_t b) {  /* float8_e4m3fn; the generator never emits NaN (0x7f/0xff) */
  const int e = (b >> 3) & 15, m = b & 7;
  const double v = e == 0 ? ldexp(m / 8.0, -6) : ldexp(1.0 + m / 8.0, e - 7);
  return (b & 0x80) ? -v : v;
}

static double half_to_double(uint16_t h) {
  const int s = h >> 15, e = (h >> 10) & 31, m = h & 1023;
  double v;
  if (e == 0) v = ldexp((double)m, -24);
  else if (e == 31) v = m ? NAN : INFINITY;
  else v = ldexp(1.0 + m / 1024.0, e - 15);
  return s ? -v : v;
}

/* One operand: rows x k codes (rows, k/2 bytes per batch) and its plain scales
 * (rows, k/16 per batch), plus the permuted layout the library reads. */
typedef struct {
  int rows, k, l;
  uint8_t* codes;  /* l * rows * k/2 */
  uint8_t* sf;     /* l * rows * k/16 (plain) */
  uint8_t* perm;   /* l * ceil(rows/128) * (k/64) * 512 */
  size_t perm_bytes;
} operand;

static void make_operand(operand* o, int rows, int k, int l) {
  const int rm = (rows + 127) / 128, rk = k / 64;
  o->rows = rows; o->k = k; o->l = l;
  o->codes = (uint8_t*)malloc((size_t)l * rows * (k / 2) + 1);
  o->sf = (uint8_t*)malloc((size_t)l * rows * (k / 16) + 1);
  o->perm_bytes = (size_t)l * rm * rk * 512;
  o->perm = (uint8_t*)calloc(o->perm_bytes + 1, 1);  /* rows past the edge keep scale 0 */
  for (size_t i = 0; i < (size_t)l * rows * (k / 2); ++i) o->codes[i] = (uint8_t)rng();
  for (int b = 0; b < l; ++b)
    for (int r = 0; r < rows; ++r)
      for (int j = 0; j < k / 16; ++j) {
        const uint8_t s = (uint8_t)(0x28 + rng() % 0x20);  /* 2^-2 .. ~2^2 */
        o->sf[((size_t)b * rows + r) * (k / 16) + j] = s;
        /* 128-row block r/128, 64-wide K block j/4: byte (r%32)*16 + ((r%128)/32)*4 + j%4 */
        const size_t atom = ((size_t)b * rm + r / 128) * rk + j / 4;
        o->perm[atom * 512 + (r % 32) * 16 + ((r % 128) / 32) * 4 + (j % 4)] = s;
      }
}

static void free_operand(operand* o) { free(o->codes); free(o->sf); free(o->perm); }

static double dot(const operand* a, int ra, const operand* b, int rb, int batch) {
  const int k = a->k;
  const uint8_t* ca = a->codes + ((size_t)batch * a->rows + ra) * (k / 2);
  const uint8_t* cb = b->codes + ((size_t)batch * b->rows + rb) * (k / 2);
  const uint8_t* sa = a->sf + ((size_t)batch * a->rows + ra) * (k / 16);
  const uint8_t* sb = b->sf + ((size_t)batch * b->rows + rb) * (k / 16);
  double acc = 0.0;
  for (int kk = 0; kk < k; ++kk) {
    const int qa = (ca[kk / 2] >> ((kk & 1) * 4)) & 15, qb = (cb[kk / 2] >> ((kk & 1) * 4)) & 15;
    acc += e2m1(qa) * e4m3(sa[kk / 16]) * e2m1(qb) * e4m3(sb[kk / 16]);
  }
  return acc;
}

static int failures = 0;
#define CHECK(cond, ...)                 \
  do {                                   \
    if (!(cond)) {                       \
      fprintf(stderr, "FAIL: " __VA_ARGS__); \
      fprintf(stderr, "\n");             \
      ++failures;                        \
    }                                    \
  } while (0)

static void* upload(const void* host, size_t bytes) {
  void* d = NULL;
  if (cudaMalloc(&d, bytes ? bytes : 16) != cudaSuccess) { fprintf(stderr, "cudaMalloc failed\n"); exit(2); }
  if (bytes) cudaMemcpy(d, host, bytes, cudaMemcpyHostToDevice);
  return d;
}

static int compare(const uint16_t* c, const operand* a, const operand* b, int l, const char* what) {
  int bad = 0;
  double worst = 0.0;
  for (int bt = 0; bt < l; ++bt)
    for (int i = 0; i < a->rows; ++i)
      for (int j = 0; j < b->rows; ++j) {
        const double exp = dot(a, i, b, j, bt);
        const double got = half_to_double(c[((size_t)bt * a->rows + i) * b->rows + j]);
        const double used = fabs(got - exp) / (1e-3 + 1e-3 * fabs(exp));  /* <= 1 passes */
        if (!(used <= 1.0)) ++bad;
        if (used > worst) worst = used;
      }
  printf("%-34s worst error %.2f of the tolerance, %d mismatches\n", what, worst, bad);
  return bad;
}

static void dense_case(int m, int n, int k, int l, int operand_order) {
  operand a, b;
  make_operand(&a, m, k, l);
  make_operand(&b, n, k, l);
  void* da = upload(a.codes, (size_t)l * m * (k / 2));
  void* db = upload(b.codes, (size_t)l * n * (k / 2));
  void* dsa = upload(a.perm, a.perm_bytes);
  void* dsb = upload(b.perm, b.perm_bytes);
  const size_t cbytes = (size_t)l * m * n * 2;
  void* dc = NULL;
  cudaMalloc(&dc, cbytes);
  cudaMemset(dc, 0xff, cbytes);  /* NaN pattern: every element must be written */
  nvfp4_options opt;
  memset(&opt, 0, sizeof(opt));
  opt.operand_order = operand_order;
  const int rc = operand_order ? nvfp4_gemm_ex(da, db, dsa, dsb, dc, m, n, k, l, NULL, &opt)
                               : nvfp4_gemm(da, db, dsa, dsb, dc, m, n, k, l, NULL);
  CHECK(rc == NVFP4_OK, "nvfp4_gemm(%d,%d,%d,%d) returned %d: %s", m, n, k, l, rc, nvfp4_last_error());
  CHECK(cudaDeviceSynchronize() == cudaSuccess, "device error after nvfp4_gemm");
  int st = -1;
  nvfp4_status_get(&st);
  CHECK(st == NVFP4_STATUS_OK, "status word %d", st);
  uint16_t* c = (uint16_t*)malloc(cbytes);
  cudaMemcpy(c, dc, cbytes, cudaMemcpyDeviceToHost);
  char what[96];
  snprintf(what, sizeof(what), "dense %dx%dx%d l=%d order=%d", m, n, k, l, operand_order);
  CHECK(compare(c, &a, &b, l, what) == 0, "%s", what);
  free(c);
  cudaFree(da); cudaFree(db); cudaFree(dsa); cudaFree(dsb); cudaFree(dc);
  free_operand(&a); free_operand(&b);
}

static void grouped_case(void) {
  enum { G = 4 };
  const int ms[G] = {96, 0, 200, 64};
  const int n = 384, k = 512;
  operand a[G], b[G];
  void *da[G], *db[G], *dsa[G], *dsb[G], *dc[G];
  int32_t sizes[G * 4];
  uint64_t abc[G * 3], sfs[G * 2];
  for (int g = 0; g < G; ++g) {
    make_operand(&a[g], ms[g], k, 1);
    make_operand(&b[g], n, k, 1);
    da[g] = upload(a[g].codes, (size_t)ms[g] * (k / 2));
    db[g] = upload(b[g].codes, (size_t)n * (k / 2));
    dsa[g] = upload(a[g].perm, a[g].perm_bytes);
    dsb[g] = upload(b[g].perm, b[g].perm_bytes);
    cudaMalloc(&dc[g], (size_t)(ms[g] ? ms[g] : 1) * n * 2);
    cudaMemset(dc[g], 0xff, (size_t)(ms[g] ? ms[g] : 1) * n * 2);
    sizes[4 * g + 0] = ms[g]; sizes[4 * g + 1] = n; sizes[4 * g + 2] = k; sizes[4 * g + 3] = 1;
    abc[3 * g + 0] = (uint64_t)(uintptr_t)da[g];
    abc[3 * g + 1] = (uint64_t)(uintptr_t)db[g];
    abc[3 * g + 2] = (uint64_t)(uintptr_t)dc[g];
    sfs[2 * g + 0] = (uint64_t)(uintptr_t)dsa[g];
    sfs[2 * g + 1] = (uint64_t)(uintptr_t)dsb[g];
  }
  void* d_sizes = upload(sizes, sizeof(sizes));
  void* d_abc = upload(abc, sizeof(abc));
  void* d_sfs = upload(sfs, sizeof(sfs));
  const size_t ws_bytes = nvfp4_grouped_gemm_workspace_size(G);
  void* ws = NULL;
  cudaMalloc(&ws, ws_bytes);
  const int rc = nvfp4_grouped_gemm((const int32_t*)d_sizes, (const uint64_t*)d_abc,
                                    (const uint64_t*)d_sfs, G, ws, ws_bytes, NULL);
  CHECK(rc == NVFP4_OK, "nvfp4_grouped_gemm returned %d: %s", rc, nvfp4_last_error());
  CHECK(cudaDeviceSynchronize() == cudaSuccess, "device error after nvfp4_grouped_gemm");
  int st = -1;
  nvfp4_status_get(&st);
  CHECK(st == NVFP4_STATUS_OK, "status word %d", st);
  for (int g = 0; g < G; ++g) {
    if (ms[g] == 0) continue;
    uint16_t* c = (uint16_t*)malloc((size_t)ms[g] * n * 2);
    cudaMemcpy(c, dc[g], (size_t)ms[g] * n * 2, cudaMemcpyDeviceToHost);
    char what[64];
    snprintf(what, sizeof(what), "grouped g=%d %dx%dx%d", g, ms[g], n, k);
    CHECK(compare(c, &a[g], &b[g], 1, what) == 0, "%s", what);
    free(c);
  }
  for (int g = 0; g < G; ++g) {
    cudaFree(da[g]); cudaFree(db[g]); cudaFree(dsa[g]); cudaFree(dsb[g]); cudaFree(dc[g]);
    free_operand(&a[g]); free_operand(&b[g]);
  }
  cudaFree(d_sizes); cudaFree(d_abc); cudaFree(d_sfs); cudaFree(ws);
}

static void error_cases(void) {
  void* p = NULL;
  cudaMalloc(&p, 1 << 20);
  int rc = nvfp4_gemm(p, p, p, p, p, 128, 128, 100, 1, NULL);
  CHECK(rc == NVFP4_ERR_UNSUPPORTED, "k = 100 gave %d", rc);
  CHECK(strlen(nvfp4_last_error()) > 0, "no message for the error");
  rc = nvfp4_gemm(NULL, p, p, p, p, 128, 128, 128, 1, NULL);
  CHECK(rc == NVFP4_ERR_INVALID_ARG, "null a gave %d", rc);
  rc = nvfp4_gemm((char*)p + 8, p, p, p, p, 128, 128, 128, 1, NULL);
  CHECK(rc == NVFP4_ERR_ALIGNMENT, "misaligned a gave %d", rc);
  rc = nvfp4_gemm(p, p, p, p, p, 0, 128, 128, 1, NULL);
  CHECK(rc == NVFP4_ERR_INVALID_ARG, "m = 0 gave %d", rc);
  printf("%-34s done\n", "argument errors");
  cudaFree(p);
}

int main(void) {
  CHECK(nvfp4_abi_version() == NVFP4_ABI_VERSION, "ABI version %d", nvfp4_abi_version());
  nvfp4_status_reset();
  dense_case(200, 320, 512, 2, 0);   /* A on the 128-row side, ragged M and N, two batches */
  dense_case(64, 384, 1024, 1, 0);   /* skinny M: B on the 128-row side (swap) */
  dense_case(130, 256, 256, 1, 2);   /* forced swap with a ragged 128-row block */
  grouped_case();
  error_cases();
  printf(failures ? "FAILED (%d)\n" : "OK\n", failures);
  return failures ? 1 : 0;
}
