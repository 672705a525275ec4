/*
 * qfn_oracle.c -- CPU restatement of the reference's quantized matrix-product
 * path.  TEST INFRASTRUCTURE ONLY: used by tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / --impl reference legs as the checker and the CPU
 * baseline.  The product (libqfn) never links, loads or calls it.
 *
 * Each function cites the reference code it restates (paths relative to the
 * reference project root).  Elementwise arithmetic is fp32 in the reference's
 * order (dequantization, scaling, SiLU, the bf16 rounding of routing
 * weights), so those results are bit-identical to the reference.  Dot
 * products accumulate in double and round once to fp32: the reference's torch
 * matmuls sum in an unspecified blocked fp32 order, so the oracle stands for
 * the exact value of the same formula and parity against it is tolerance-based.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define HID 2560
#define INTER 640
#define BLOCK 2764800L
#define O_GW 0L
#define O_UW 819200L
#define O_DW 1638400L
#define O_GS 2457600L
#define O_US 2560000L
#define O_DS 2662400L

/* qmoe.py:87 -- e2m1 code -> value; bit 3 is the sign (code 8 is -0). */
static const float E2M1[16] = {0.f, .5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f,
                               -0.f, -.5f, -1.f, -1.5f, -2.f, -3.f, -4.f, -6.f};

int oracle_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
  return omp_get_max_threads();
#else
  (void)n;
  return 1;
#endif
}

/* float8_e4m3fn byte -> fp32 (the decode torch.float8_e4m3fn performs in
 * qmoe.py:101, qwen_engine.py:83 and tests/test_gemv.py:9): sign, 4-bit
 * exponent with bias 7, 3-bit mantissa; exponent 0 is subnormal (m * 2^-9);
 * S.1111.111 is NaN; there are no infinities. */
float oracle_e4m3_to_f32(uint8_t b) {
  const int sgn = b >> 7, e = (b >> 3) & 15, m = b & 7;
  float v;
  if (e == 15 && m == 7) return NAN;
  if (e == 0) v = ldexpf((float)m, -9);
  else v = ldexpf(1.0f + (float)m / 8.0f, e - 7);
  return sgn ? -v : v;
}

/* fp32 -> float8_e4m3fn byte, round to nearest even (the conversion
 * `.to(torch.float8_e4m3fn)` in to_fp8_rows, qwen_engine.py:64).  The e4m3
 * grid is extended with 480 (the pattern that e4m3fn reserves for NaN); a
 * value that rounds to >= 480 in magnitude, or is NaN, gives 0x7f | sign. */
uint8_t oracle_f32_to_e4m3(float f) {
  uint8_t sgn = signbit(f) ? 0x80 : 0;
  float a = fabsf(f);
  if (isnan(f)) return 0x7f | sgn;
  if (a == 0.f) return sgn;
  int e2;
  frexpf(a, &e2);           /* a = fr * 2^e2, fr in [0.5, 1) -> a in [2^(e2-1), 2^e2) */
  int ex = e2 - 1;          /* unbiased exponent of a */
  if (ex < -6) ex = -6;     /* subnormal range shares the 2^-9 quantum */
  const float quantum = ldexpf(1.0f, ex - 3);
  float q = a / quantum;    /* exact: power-of-two division */
  float r = rintf(q);       /* round half to even (default FP environment) */
  float v = r * quantum;
  if (v >= 480.f) return 0x7f | sgn;
  /* re-encode v (exactly representable on the extended grid) */
  if (v == 0.f) return sgn;
  int e3;
  frexpf(v, &e3);
  int ue = e3 - 1;
  if (ue < -6) { /* subnormal: v = m * 2^-9 */
    int m = (int)ldexpf(v, 9);
    return sgn | (uint8_t)m;
  }
  int m = (int)(ldexpf(v, -ue) * 8.0f) - 8;
  return sgn | (uint8_t)(((ue + 7) << 3) | m);
}

/* qmoe.deq (qmoe.py:93-102): out[n][k] = E2M1[nib] * e4m3(s[n][k/16]) * ws2,
 * low nibble = even k (qmoe.py:96-100); swap != 0 is the reference's SWAP
 * negative control (qmoe.py:90,98-99). */
void oracle_deq(const uint8_t* w, const uint8_t* s, float ws2, float* out, long N, long K, int swap) {
  const long kb = K / 2, kg = K / 16;
#pragma omp parallel for schedule(static)
  for (long n = 0; n < N; ++n) {
    for (long k = 0; k < K; ++k) {
      const uint8_t byte = w[n * kb + k / 2];
      int nib = (k & 1) ? (byte >> 4) : (byte & 15);
      if (swap) nib = (k & 1) ? (byte & 15) : (byte >> 4);
      const float sc = oracle_e4m3_to_f32(s[n * kg + k / 16]);
      volatile float t = E2M1[nib] * sc; /* w * s, then * ws2 (left to right) */
      out[n * K + k] = t * ws2;
    }
  }
}

/* qmoe.block_deq (qmoe.py:105-111). */
void oracle_block_deq(const uint8_t* blk, const float* s2, float* g, float* u, float* d) {
  oracle_deq(blk + O_GW, blk + O_GS, s2[0], g, INTER, HID, 0);
  oracle_deq(blk + O_UW, blk + O_US, s2[1], u, INTER, HID, 0);
  oracle_deq(blk + O_DW, blk + O_DS, s2[2], d, HID, INTER, 0);
}

static float silu(float v) { return v / (1.0f + expf(-v)); } /* F.silu / qmoe.py:50 */

/* The moe_decode reference of tests/test_qmoe.py:24-28:
 *   ref = sum_j coef[j] * (d_j @ (silu(g_j @ x) * (u_j @ x)))     in fp32,
 * with (g, u, d) = block_deq(block of sidx[j], s2[j]).  out[2560]; if h is
 * non-null it receives h[j][640]. */
void oracle_moe_decode(const uint8_t* table, const int32_t* sidx, const float* s2, const float* coef,
                       const float* x, int K, float* out, float* h) {
  float* G = (float*)malloc(sizeof(float) * INTER * HID);
  float* U = (float*)malloc(sizeof(float) * INTER * HID);
  float* D = (float*)malloc(sizeof(float) * HID * INTER);
  float* hj = (float*)malloc(sizeof(float) * INTER);
  for (long r = 0; r < HID; ++r) out[r] = 0.f;
  for (int j = 0; j < K; ++j) {
    oracle_block_deq(table + (long)sidx[j] * BLOCK, s2 + 3 * j, G, U, D);
#pragma omp parallel for schedule(static)
    for (long n = 0; n < INTER; ++n) {
      double ag = 0.0, au = 0.0;
      for (long k = 0; k < HID; ++k) {
        ag += (double)G[n * HID + k] * x[k];
        au += (double)U[n * HID + k] * x[k];
      }
      hj[n] = silu((float)ag) * (float)au;
    }
    if (h) memcpy(h + (long)j * INTER, hj, sizeof(float) * INTER);
#pragma omp parallel for schedule(static)
    for (long r = 0; r < HID; ++r) {
      double a = 0.0;
      for (long n = 0; n < INTER; ++n) a += (double)D[r * INTER + n] * hj[n];
      out[r] += coef[j] * (float)a;
    }
  }
  free(G); free(U); free(D); free(hj);
}

/* to_fp8_rows (qwen_engine.py:59-64): s = max(rowmax|w| / 448, 1e-12),
 * q = e4m3(w / s), all in fp32. */
void oracle_to_fp8_rows(const float* w, long N, long K, uint8_t* q, float* s) {
#pragma omp parallel for schedule(static)
  for (long n = 0; n < N; ++n) {
    float amax = 0.f;
    for (long k = 0; k < K; ++k) {
      float a = fabsf(w[n * K + k]);
      if (a > amax || isnan(a)) amax = a;
    }
    float sc = amax / 448.0f;
    if (sc < 1e-12f) sc = 1e-12f;
    s[n] = sc;
    for (long k = 0; k < K; ++k) q[n * K + k] = oracle_f32_to_e4m3(w[n * K + k] / sc);
  }
}

/* The gemv reference of tests/test_gemv.py:9: y = (q.float() * s[:,None]) @
 * x.float(), fp32 (before the bf16 output rounding of fp8gemv.py:17). */
void oracle_gemv(const uint8_t* q, const float* s, const float* x, long N, long K, float* y) {
#pragma omp parallel for schedule(static)
  for (long n = 0; n < N; ++n) {
    double a = 0.0;
    for (long k = 0; k < K; ++k) {
      volatile float wq = oracle_e4m3_to_f32(q[n * K + k]) * s[n];
      a += (double)wq * x[k];
    }
    y[n] = (float)a;
  }
}

/* The prefill expert loop of QwenEngine.moe (qwen_engine.py:835-852):
 *   for e in sorted(distinct experts of layer):
 *     tok, slot = where(ti == e)
 *     h = silu(x[tok] @ g.T) * (x[tok] @ u.T)
 *     out.index_add_(tok, (h @ d.T) * tv[tok, slot])
 * x f32[T][2560] (already .float()), ti int32[T][topk] expert ids of this
 * layer, tv f32[T][topk] (the bf16 routing weights as fp32), table + base:
 * block of expert e is table[(base + e) * BLOCK], s2l f32[n_experts][3].
 * out f32[T][2560] (zeroed here). */
void oracle_moe_prefill(const float* x, long T, const int32_t* ti, const float* tv, int topk,
                        const uint8_t* table, long base, const float* s2l, int n_experts, float* out) {
  float* G = (float*)malloc(sizeof(float) * INTER * HID);
  float* U = (float*)malloc(sizeof(float) * INTER * HID);
  float* D = (float*)malloc(sizeof(float) * HID * INTER);
  long* tok = (long*)malloc(sizeof(long) * T * topk);
  float* w = (float*)malloc(sizeof(float) * T * topk);
  float* H = (float*)malloc(sizeof(float) * T * topk * INTER);
  memset(out, 0, sizeof(float) * T * HID);
  for (int e = 0; e < n_experts; ++e) {
    long m = 0;
    for (long t = 0; t < T; ++t)
      for (int k = 0; k < topk; ++k)
        if (ti[t * topk + k] == e) { tok[m] = t; w[m] = tv[t * topk + k]; ++m; }
    if (!m) continue;
    oracle_block_deq(table + (base + e) * BLOCK, s2l + 3 * e, G, U, D);
#pragma omp parallel for schedule(static)
    for (long i = 0; i < m; ++i) {
      const float* xr = x + tok[i] * HID;
      for (long n = 0; n < INTER; ++n) {
        double ag = 0.0, au = 0.0;
        for (long k = 0; k < HID; ++k) { ag += (double)xr[k] * G[n * HID + k]; au += (double)xr[k] * U[n * HID + k]; }
        H[i * INTER + n] = silu((float)ag) * (float)au;
      }
    }
    /* index_add_: contributions of expert e land in pair order.  Threads own
     * output columns r, so a token routed to e twice accumulates without a
     * race, in the same order as torch's CPU index_add_. */
#pragma omp parallel for schedule(static)
    for (long r = 0; r < HID; ++r) {
      for (long i = 0; i < m; ++i) {
        double a = 0.0;
        for (long n = 0; n < INTER; ++n) a += (double)H[i * INTER + n] * D[r * INTER + n];
        out[tok[i] * HID + r] += (float)a * w[i];
      }
    }
  }
  free(G); free(U); free(D); free(tok); free(w); free(H);
}

/* The router of QwenEngine.moe (qwen_engine.py:803-806) for fp32 logits:
 * probs = softmax(logits) in fp32; top-`topk` by probability (ties -> lower
 * index first); tv = probs_top / sum(probs_top); coef = bf16(tv) returned as
 * its fp32 value.  logits f32[T][E]; ti int32[T][topk]; coef f32[T][topk]. */
static float bf16_round(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7f800000u) == 0x7f800000u) { /* inf / nan */
    if (u & 0x7fffffu) u |= 0x400000u;
    u &= 0xffff0000u;
  } else {
    u += 0x7fffu + ((u >> 16) & 1u);
    u &= 0xffff0000u;
  }
  memcpy(&f, &u, 4);
  return f;
}

void oracle_route(const float* logits, long T, int E, int topk, int32_t* ti, float* coef) {
#pragma omp parallel for schedule(static)
  for (long t = 0; t < T; ++t) {
    const float* l = logits + t * E;
    float mx = -INFINITY;
    for (int e = 0; e < E; ++e) mx = l[e] > mx ? l[e] : mx;
    float* p = (float*)malloc(sizeof(float) * E);
    float sum = 0.f;
    for (int e = 0; e < E; ++e) { p[e] = expf(l[e] - mx); sum += p[e]; }
    for (int e = 0; e < E; ++e) p[e] /= sum;
    char* used = (char*)calloc(E, 1);
    float tsum = 0.f;
    float* tvv = (float*)malloc(sizeof(float) * topk);
    for (int k = 0; k < topk; ++k) {
      int best = -1;
      for (int e = 0; e < E; ++e)
        if (!used[e] && (best < 0 || p[e] > p[best])) best = e;
      used[best] = 1;
      ti[t * topk + k] = best;
      tvv[k] = p[best];
    }
    for (int k = 0; k < topk; ++k) tsum += tvv[k];
    for (int k = 0; k < topk; ++k) coef[t * topk + k] = bf16_round(tvv[k] / tsum);
    free(p); free(used); free(tvv);
  }
}
