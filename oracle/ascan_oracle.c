/*
 * ascan_oracle.c -- CPU restatement of the reference's scan semantics.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product links, loads or calls this
 * file: it is the checker used by tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py.
 *
 * Every routine computes in IEEE double precision, sequentially, one
 * (channel, sequence) pair at a time, following the reference's gold label and
 * its hand-derived backward:
 *
 *   forward (causal)      h[t] = g[t] * h[t-1] + x[t],  h[start-1] := 0
 *     reference: tests/test_scan_dtypes.py:26-38 (sequential_scan_gold),
 *                identical copy at bench/bench_accuracy.py:40-49.
 *   forward (reverse)     h[t] = g[t] * h[t+1] + x[t],  h[end] := 0
 *     reference: tests/test_scan_kernels.py:281-286 (expected values),
 *                tests/test_scan_dtypes.py:173-177 (flip / scan / flip).
 *   cumulative gate product (the TESTING write-back of the forward kernels)
 *                         a[t] = prod_{s=start..t} g[s]   (reverse: t..end-1)
 *     reference: src/associative_scan_triton/_kernels.py:74-76, :161-163,
 *                golden values tests/test_scan_kernels.py:149-151, :202-204.
 *   backward of the causal scan (CAUSAL=True)
 *                         dh[t] = dy[t] + g[t+1] * dh[t+1],  g[end] := 1
 *                         dx[t] = dh[t],  dg[t] = dh[t] * h[t-1],  h[start-1] := 0
 *     reference: tests/test_scan_kernels.py:850-897 (derivation),
 *                src/associative_scan_triton/_kernels.py:184-196.
 *   backward of the reverse scan (CAUSAL=False) mirrors it:
 *                         dh[t] = dy[t] + g[t-1] * dh[t-1],  g[start-1] := 1
 *                         dx[t] = dh[t],  dg[t] = dh[t] * h[t+1],  h[end] := 0
 *     reference: src/associative_scan_triton/_kernels.py:191-194.
 *   shift_pad             out[t] = pad at sequence heads (shift right) or
 *                         tails (shift left), else data[t -/+ 1]
 *     reference: src/associative_scan_triton/_shift_pad.py:18-55 (torch.roll
 *                variant, wrap-around) and :63-118 (kernel variant, clamped).
 *
 * Layout (reference src/associative_scan_triton/scan_eager.py:74-83): every
 * tensor is [C, BL] row-major; sequence i of channel c occupies
 * [c*BL + cu[i], c*BL + cu[i+1]).  Positions of a row that lie in no
 * sequence (t < cu[0]) are left untouched, as the reference's masked stores
 * leave them.  Inputs are float32 (fp16/bf16 values convert to float32
 * exactly); outputs are float64.
 */
#include <stddef.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORACLE_API __attribute__((visibility("default")))

static int64_t clamp64(int64_t v, int64_t lo, int64_t hi) {
  return v < lo ? lo : (v > hi ? hi : v);
}

static void set_threads(int nthreads) {
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#else
  (void)nthreads;
#endif
}

ORACLE_API int oracle_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* Forward scan.  gprod may be NULL (no cumulative gate product wanted). */
ORACLE_API void oracle_scan_fwd(const float *g, const float *x, double *y,
                                double *gprod, const int64_t *cu, int64_t S,
                                int64_t C, int64_t BL, int reverse,
                                int nthreads) {
  set_threads(nthreads);
#pragma omp parallel for schedule(static)
  for (int64_t c = 0; c < C; ++c) {
    const float *gr = g + c * BL;
    const float *xr = x + c * BL;
    double *yr = y + c * BL;
    double *pr = gprod ? gprod + c * BL : NULL;
    for (int64_t i = 0; i < S; ++i) {
      int64_t s = clamp64(cu[i], 0, BL), e = clamp64(cu[i + 1], 0, BL);
      if (e <= s) continue;
      if (!reverse) {
        double h = (double)xr[s], a = (double)gr[s];
        yr[s] = h;
        if (pr) pr[s] = a;
        for (int64_t t = s + 1; t < e; ++t) {
          double gt = (double)gr[t];
          h = gt * h + (double)xr[t];
          a = a * gt;
          yr[t] = h;
          if (pr) pr[t] = a;
        }
      } else {
        double h = (double)xr[e - 1], a = (double)gr[e - 1];
        yr[e - 1] = h;
        if (pr) pr[e - 1] = a;
        for (int64_t t = e - 2; t >= s; --t) {
          double gt = (double)gr[t];
          h = gt * h + (double)xr[t];
          a = a * gt;
          yr[t] = h;
          if (pr) pr[t] = a;
        }
      }
    }
  }
}

/* Backward of a forward scan; causal=1 is the adjoint of the causal scan,
 * causal=0 the adjoint of the reverse scan.  h holds the forward outputs. */
ORACLE_API void oracle_scan_bwd(const float *dy, const float *g,
                                const float *h, double *dx, double *dg,
                                const int64_t *cu, int64_t S, int64_t C,
                                int64_t BL, int causal, int nthreads) {
  set_threads(nthreads);
#pragma omp parallel for schedule(static)
  for (int64_t c = 0; c < C; ++c) {
    const float *dyr = dy + c * BL;
    const float *gr = g + c * BL;
    const float *hr = h + c * BL;
    double *dxr = dx + c * BL;
    double *dgr = dg + c * BL;
    for (int64_t i = 0; i < S; ++i) {
      int64_t s = clamp64(cu[i], 0, BL), e = clamp64(cu[i + 1], 0, BL);
      if (e <= s) continue;
      if (causal) {
        double d = 0.0;
        for (int64_t t = e - 1; t >= s; --t) {
          d = (t == e - 1) ? (double)dyr[t] : (double)gr[t + 1] * d + (double)dyr[t];
          dxr[t] = d;
          dgr[t] = (t == s) ? 0.0 : d * (double)hr[t - 1];
        }
      } else {
        double d = 0.0;
        for (int64_t t = s; t < e; ++t) {
          d = (t == s) ? (double)dyr[t] : (double)gr[t - 1] * d + (double)dyr[t];
          dxr[t] = d;
          dgr[t] = (t == e - 1) ? 0.0 : d * (double)hr[t + 1];
        }
      }
    }
  }
}

/* Same as the two routines above but with the forward states computed here in
 * float64 from g and x (the "true" gradient of sum(y * dy)). */
ORACLE_API void oracle_scan_fwd_bwd(const float *g, const float *x,
                                    const float *dy, double *y, double *dx,
                                    double *dg, const int64_t *cu, int64_t S,
                                    int64_t C, int64_t BL, int causal,
                                    int nthreads) {
  set_threads(nthreads);
#pragma omp parallel for schedule(static)
  for (int64_t c = 0; c < C; ++c) {
    const float *gr = g + c * BL;
    const float *xr = x + c * BL;
    const float *dyr = dy + c * BL;
    double *yr = y + c * BL;
    double *dxr = dx + c * BL;
    double *dgr = dg + c * BL;
    for (int64_t i = 0; i < S; ++i) {
      int64_t s = clamp64(cu[i], 0, BL), e = clamp64(cu[i + 1], 0, BL);
      if (e <= s) continue;
      if (causal) {
        double hh = 0.0;
        for (int64_t t = s; t < e; ++t) {
          hh = (t == s) ? (double)xr[t] : (double)gr[t] * hh + (double)xr[t];
          yr[t] = hh;
        }
        double d = 0.0;
        for (int64_t t = e - 1; t >= s; --t) {
          d = (t == e - 1) ? (double)dyr[t] : (double)gr[t + 1] * d + (double)dyr[t];
          dxr[t] = d;
          dgr[t] = (t == s) ? 0.0 : d * yr[t - 1];
        }
      } else {
        double hh = 0.0;
        for (int64_t t = e - 1; t >= s; --t) {
          hh = (t == e - 1) ? (double)xr[t] : (double)gr[t] * hh + (double)xr[t];
          yr[t] = hh;
        }
        double d = 0.0;
        for (int64_t t = s; t < e; ++t) {
          d = (t == s) ? (double)dyr[t] : (double)gr[t - 1] * d + (double)dyr[t];
          dxr[t] = d;
          dgr[t] = (t == e - 1) ? 0.0 : d * yr[t + 1];
        }
      }
    }
  }
}

/* shift_pad.  backward=1 shifts right (out[t] = data[t-1], pad at sequence
 * starts cu[0..S-1]); backward=0 shifts left (out[t] = data[t+1], pad at
 * sequence ends cu[1..S]-1).  wrap=1 follows the torch.roll variant (the
 * source index wraps around the row), wrap=0 the kernel variant (the source
 * index is clamped to [0, BL-1]).  Every output position is written. */
ORACLE_API void oracle_shift_pad(const float *data, double *out,
                                 const int64_t *cu, int64_t S, int64_t C,
                                 int64_t BL, double pad_value, int backward,
                                 int wrap, int nthreads) {
  set_threads(nthreads);
  if (BL <= 0) return;
#pragma omp parallel for schedule(static)
  for (int64_t c = 0; c < C; ++c) {
    const float *dr = data + c * BL;
    double *orow = out + c * BL;
    for (int64_t t = 0; t < BL; ++t) {
      int64_t src = backward ? t - 1 : t + 1;
      if (wrap)
        src = (src % BL + BL) % BL;
      else
        src = clamp64(src, 0, BL - 1);
      orow[t] = (double)dr[src];
    }
    for (int64_t i = 0; i < S; ++i) {
      int64_t b = backward ? cu[i] : cu[i + 1] - 1;
      if (b >= 0 && b < BL) orow[b] = pad_value;
    }
  }
}
