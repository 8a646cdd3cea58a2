/*
 * CPU restatement of the HCLSM Level-0 selective scan (forward and backward).
 *
 * TEST INFRASTRUCTURE ONLY: this file is the parity checker and the timed CPU
 * baseline.  Nothing in the product path links or calls it.
 *
 * Forward follows hclsm/kernels/ssm_scan_kernel.py:
 *   clamp=1  -> sequential_ssm_scan            (:42-86)
 *              A = -clamp(exp(A_log), 1e-6, 1); dt clamped to [1e-3, 1];
 *              dA = exp(clamp(dt*A, -20, 0))
 *   clamp=0  -> parallel_ssm_scan_pytorch / the Triton forward (:168-218, :227-290)
 *              A = -exp(A_log); dA = exp(dt*A)
 *   per t:  h = dA*h + (dt*B)*x ;  y = sum_s h*C
 * Optional extensions (no reference counterpart inside the scan op; the gate
 * form follows hclsm/dynamics/level0_ssm.py:73,104):
 *   y_out = (y + D*x) * silu(z)        (D and z may each be NULL)
 *
 * Backward restates _TritonSSMScan.backward (ssm_scan_kernel.py:321-377) for
 * clamp=0, and the autograd of sequential_ssm_scan for clamp=1 (clamp gradients
 * pass where min <= v <= max, as torch.clamp's backward does).
 *
 * Functions are single-threaded over the sequences they are given; the Python
 * wrapper (oracle/scan.py) splits sequences across host threads.
 *
 * All arrays are fp32, row-major: x, dt, y (nseq, L, Dn); B, C (nseq, L, S);
 * A_log (Dn, S); D (Dn); z (nseq, L, Dn).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static inline float clampf(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }
static inline float sigmoidf_(float v) { return 1.0f / (1.0f + expf(-v)); }

void oracle_scan_fwd(const float* x, const float* dt, const float* A_log, const float* B,
                     const float* C, const float* Dv, const float* z, float* y, int64_t nseq,
                     int L, int Dn, int S, int clamp) {
  for (int64_t bd = 0; bd < nseq * (int64_t)Dn; ++bd) {
    const int64_t b = bd / Dn;
    const int d = (int)(bd % Dn);
    float A[64], h[64];
    for (int s = 0; s < S; ++s) {
      float e = expf(A_log[(int64_t)d * S + s]);
      if (clamp) e = clampf(e, 1e-6f, 1.0f);
      A[s] = -e;
      h[s] = 0.0f;
    }
    for (int t = 0; t < L; ++t) {
      const int64_t i = (b * L + t) * (int64_t)Dn + d;
      const float* Bt = B + (b * L + t) * (int64_t)S;
      const float* Ct = C + (b * L + t) * (int64_t)S;
      float dtv = dt[i];
      if (clamp) dtv = clampf(dtv, 1e-3f, 1.0f);
      const float xv = x[i];
      float acc = 0.0f;
      for (int s = 0; s < S; ++s) {
        float u = dtv * A[s];
        if (clamp) u = clampf(u, -20.0f, 0.0f);
        const float dA = expf(u);
        h[s] = dA * h[s] + (dtv * Bt[s]) * xv;
        acc += h[s] * Ct[s];
      }
      if (Dv) acc += Dv[d] * xv;
      if (z) {
        const float zv = z[i];
        acc *= zv * sigmoidf_(zv);
      }
      y[i] = acc;
    }
  }
}

/*
 * Backward over sequences [0, nseq) of the given arrays.  dy is the upstream
 * gradient of y_out.  Outputs (overwritten): dx, ddt (nseq, L, Dn); dB, dC
 * (nseq, L, S); dz (nseq, L, Dn) if z.  Accumulated (+=, double):
 *   gA (Dn, S) = sum over (seq, t) of dL/dA (the caller multiplies by dA/dA_log)
 *   gD (Dn)    = dL/dD
 */
void oracle_scan_bwd(const float* x, const float* dt, const float* A_log, const float* B,
                     const float* C, const float* Dv, const float* z, const float* dy, float* dx,
                     float* ddt, float* dB, float* dC, float* dz, double* gA, double* gD,
                     int64_t nseq, int L, int Dn, int S, int clamp) {
  memset(dB, 0, sizeof(float) * (size_t)nseq * L * S);
  memset(dC, 0, sizeof(float) * (size_t)nseq * L * S);
  float* hs = (float*)malloc(sizeof(float) * (size_t)(L + 1) * S);
  float* dAs = (float*)malloc(sizeof(float) * (size_t)L * S);
  float* mu = (float*)malloc(sizeof(float) * (size_t)L * S);
  for (int64_t b = 0; b < nseq; ++b) {
    for (int d = 0; d < Dn; ++d) {
      float A[64];
      for (int s = 0; s < S; ++s) {
        float e = expf(A_log[(int64_t)d * S + s]);
        if (clamp) e = clampf(e, 1e-6f, 1.0f);
        A[s] = -e;
      }
      /* forward recompute: hs[t+1] = state after step t */
      for (int s = 0; s < S; ++s) hs[s] = 0.0f;
      for (int t = 0; t < L; ++t) {
        const int64_t i = (b * L + t) * (int64_t)Dn + d;
        const float* Bt = B + (b * L + t) * (int64_t)S;
        float dtv = dt[i];
        if (clamp) dtv = clampf(dtv, 1e-3f, 1.0f);
        for (int s = 0; s < S; ++s) {
          float u = dtv * A[s];
          float m = 1.0f;
          if (clamp) {
            m = (u >= -20.0f && u <= 0.0f) ? 1.0f : 0.0f;
            u = clampf(u, -20.0f, 0.0f);
          }
          const float dA = expf(u);
          dAs[t * S + s] = dA;
          mu[t * S + s] = m;
          hs[(t + 1) * S + s] = dA * hs[t * S + s] + (dtv * Bt[s]) * x[i];
        }
      }
      /* reverse pass */
      float g[64];
      for (int s = 0; s < S; ++s) g[s] = 0.0f;
      for (int t = L - 1; t >= 0; --t) {
        const int64_t i = (b * L + t) * (int64_t)Dn + d;
        const float* Bt = B + (b * L + t) * (int64_t)S;
        const float* Ct = C + (b * L + t) * (int64_t)S;
        float* dBt = dB + (b * L + t) * (int64_t)S;
        float* dCt = dC + (b * L + t) * (int64_t)S;
        const float dt_raw = dt[i];
        float dtv = dt_raw;
        float mdt = 1.0f;
        if (clamp) {
          mdt = (dt_raw >= 1e-3f && dt_raw <= 1.0f) ? 1.0f : 0.0f;
          dtv = clampf(dt_raw, 1e-3f, 1.0f);
        }
        const float xv = x[i];
        float gy = dy[i];
        if (z) {
          float yscan = 0.0f;
          for (int s = 0; s < S; ++s) yscan += hs[(t + 1) * S + s] * Ct[s];
          const float zv = z[i];
          const float sg = sigmoidf_(zv);
          const float pre = yscan + (Dv ? Dv[d] * xv : 0.0f);
          dz[i] = gy * pre * sg * (1.0f + zv * (1.0f - sg));
          gy = gy * zv * sg;
        }
        float gx = 0.0f, gdt = 0.0f;
        if (Dv) {
          gx += gy * Dv[d];
          gD[d] += (double)gy * xv;
        }
        for (int s = 0; s < S; ++s) {
          g[s] += gy * Ct[s];
          dCt[s] += gy * hs[(t + 1) * S + s];
          const float hp = hs[t * S + s];
          const float dA = dAs[t * S + s];
          const float gdA = g[s] * hp * mu[t * S + s];
          gdt += gdA * dA * A[s];
          gA[d * S + s] += (double)(gdA * dA * dtv);
          gx += g[s] * dtv * Bt[s];
          gdt += g[s] * Bt[s] * xv;
          dBt[s] += g[s] * dtv * xv;
          g[s] = g[s] * dA;
        }
        dx[i] = gx;
        ddt[i] = gdt * mdt;
      }
    }
  }
  free(hs); free(dAs); free(mu);
}
