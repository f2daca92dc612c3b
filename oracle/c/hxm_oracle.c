/*
 * hxm_oracle.c — plain-C restatement of the reference's recurrent loops.
 *
 * TEST INFRASTRUCTURE ONLY: used by the tests as a fast checker on slices of
 * large workloads and by bench.py as the timed CPU baseline / reference arm.
 * The product library never links or calls it.
 *
 * Arithmetic is fp32 like the reference's own loops (which keep their state
 * in the input dtype); libm expf/log1pf/tanhf.  Independent channels / heads
 * run in parallel with OpenMP (the reference's torch loops are likewise
 * vectorised over batch x channels and threaded by torch's intra-op pool).
 *
 * Functions and the reference code they restate:
 *   hxm_oracle_scan      selective_scan_pytorch
 *                        (hybrid_xmamba/kernels/selective_scan/scan_interface.py:103-152),
 *                        ZOH rule of scan_triton.py:135-160, gates of
 *                        scan_interface.py:57-58 (y*z) and mamba_block.py:130 (y*silu(z)),
 *                        softplus(dt + bias) of mamba_block.py:115-116
 *   hxm_oracle_mlstm     tfla_forward_pytorch (hybrid_xmamba/kernels/tfla/tfla_interface.py:84-139)
 *   hxm_oracle_slstm     the loop of sLSTMBlock.forward (hybrid_xmamba/layers/slstm_block.py:91-127)
 *                        plus the optional block-diagonal recurrent term R
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

void hxm_oracle_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

int hxm_oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

static float softplusf(float x) { return x > 20.f ? x : log1pf(expf(x)); }
static float sigmoidf_(float x) { return 1.f / (1.f + expf(-x)); }

/*
 * Selective scan, time-major layout:
 *   u, dt, z, y : (batch, dim, seqlen)      B, C : (batch, dstate, seqlen)
 *   A : (dim, dstate)   D, bias : (dim) or NULL   h0, hT : (batch, dim, dstate) or NULL
 *   z_mode 0 none / 1 y*z / 2 y*silu(z);  disc 0 euler / 1 zoh
 */
void hxm_oracle_scan(int batch, int seqlen, int dim, int dstate, const float* u, const float* dt,
                     const float* A, const float* B, const float* C, const float* D, const float* z,
                     const float* bias, int softplus, int z_mode, int disc, const float* h0, float* y,
                     float* hT) {
#pragma omp parallel for schedule(static)
  for (int64_t bd = 0; bd < (int64_t)batch * dim; ++bd) {
    const int b = (int)(bd / dim), d = (int)(bd % dim);
    float h[256];
    const float* a = A + (int64_t)d * dstate;
    for (int n = 0; n < dstate; ++n) h[n] = h0 ? h0[bd * dstate + n] : 0.f;
    const float* ub = u + bd * seqlen;
    const float* db = dt + bd * seqlen;
    const float* zb = z ? z + bd * seqlen : NULL;
    float* yb = y + bd * seqlen;
    const float* Bb = B + (int64_t)b * dstate * seqlen;
    const float* Cb = C + (int64_t)b * dstate * seqlen;
    const float Dd = D ? D[d] : 0.f, bi = bias ? bias[d] : 0.f;
    for (int t = 0; t < seqlen; ++t) {
      float dl = db[t] + bi;
      if (softplus) dl = softplusf(dl);
      const float x = ub[t];
      float acc = 0.f;
      for (int n = 0; n < dstate; ++n) {
        const float dA = dl * a[n];
        const float Ab = expf(dA);
        const float bt = Bb[(int64_t)n * seqlen + t];
        float Bbar;
        if (disc == 1 && fabsf(dA) >= 0.01f) Bbar = (Ab - 1.f) / a[n] * bt;
        else Bbar = dl * bt;
        h[n] = Ab * h[n] + Bbar * x;
        acc += h[n] * Cb[(int64_t)n * seqlen + t];
      }
      acc += Dd * x;
      if (z_mode == 1) acc *= zb[t];
      else if (z_mode == 2) acc *= zb[t] * sigmoidf_(zb[t]);
      yb[t] = acc;
    }
    if (hT)
      for (int n = 0; n < dstate; ++n) hT[bd * dstate + n] = h[n];
  }
}

/*
 * mLSTM recurrence (reference semantics, no stabilizer):
 *   q, k : (BH, L, dk)   v, h : (BH, L, dv)   gates i, f ACTIVATED, (BH, L) if
 *   per_channel == 0 else (BH, L, dk).  C : (BH, dk, dv), n : (BH, dk) in/out
 *   (zero-initialised by the caller for a fresh sequence).
 */
void hxm_oracle_mlstm(int BH, int L, int dk, int dv, const float* q, const float* k, const float* v,
                      const float* ig, const float* fg, int per_channel, float* h, float* C, float* n) {
#pragma omp parallel for schedule(dynamic, 1)
  for (int bh = 0; bh < BH; ++bh) {
    float* Cs = C + (int64_t)bh * dk * dv;
    float* ns = n + (int64_t)bh * dk;
    float* num = (float*)malloc(sizeof(float) * dv);
    for (int t = 0; t < L; ++t) {
      const float* qt = q + ((int64_t)bh * L + t) * dk;
      const float* kt = k + ((int64_t)bh * L + t) * dk;
      const float* vt = v + ((int64_t)bh * L + t) * dv;
      const float* it = per_channel ? ig + ((int64_t)bh * L + t) * dk : ig + (int64_t)bh * L + t;
      const float* ft = per_channel ? fg + ((int64_t)bh * L + t) * dk : fg + (int64_t)bh * L + t;
      float den = 0.f;
      for (int e = 0; e < dv; ++e) num[e] = 0.f;
      for (int j = 0; j < dk; ++j) {
        const float fj = per_channel ? ft[j] : ft[0];
        const float ij = per_channel ? it[j] : it[0];
        const float ikj = ij * kt[j];
        float* row = Cs + (int64_t)j * dv;
        const float qj = qt[j];
        for (int e = 0; e < dv; ++e) {
          row[e] = fj * row[e] + ikj * vt[e];
          num[e] += qj * row[e];
        }
        ns[j] = fj * ns[j] + ikj;
        den += qj * ns[j];
      }
      if (den < 1.f) den = 1.f;
      float* ht = h + ((int64_t)bh * L + t) * dv;
      for (int e = 0; e < dv; ++e) ht[e] = num[e] / den;
    }
    free(num);
  }
}

/*
 * sLSTM recurrence:
 *   g : (batch, L, heads, 4, hd) pre-activations [i|f|o|c~]; R : (heads, hd, 4*hd) or NULL;
 *   w : (hd); h_out : (batch, L, heads, hd); hs, cs : (batch, heads, hd) in/out (true cell).
 */
void hxm_oracle_slstm(int batch, int L, int heads, int hd, const float* g, const float* R, const float* w,
                      float eps, int exp_gate, float* h_out, float* hs, float* cs) {
#pragma omp parallel for schedule(dynamic, 1)
  for (int bh = 0; bh < batch * heads; ++bh) {
    const int b = bh / heads, hh = bh % heads;
    float* hv = hs + (int64_t)bh * hd;
    float* cv = cs + (int64_t)bh * hd;
    float* pre = (float*)malloc(sizeof(float) * 4 * hd);
    const float* Rh = R ? R + (int64_t)hh * hd * 4 * hd : NULL;
    for (int t = 0; t < L; ++t) {
      const float* gt = g + (((int64_t)b * L + t) * heads + hh) * 4 * hd;
      for (int c = 0; c < 4 * hd; ++c) pre[c] = gt[c];
      if (Rh)
        for (int j = 0; j < hd; ++j) {
          const float hj = hv[j];
          const float* r = Rh + (int64_t)j * 4 * hd;
          for (int c = 0; c < 4 * hd; ++c) pre[c] += hj * r[c];
        }
      float ss = 0.f;
      for (int j = 0; j < hd; ++j) {
        const float ig = exp_gate ? expf(pre[j]) : sigmoidf_(pre[j]);
        const float fg = sigmoidf_(pre[hd + j]);
        cv[j] = fg * cv[j] + ig * tanhf(pre[3 * hd + j]);
        ss += cv[j] * cv[j];
      }
      const float rinv = 1.f / sqrtf(ss / hd + eps);
      float* ht = h_out + (((int64_t)b * L + t) * heads + hh) * hd;
      for (int j = 0; j < hd; ++j) {
        const float og = sigmoidf_(pre[2 * hd + j]);
        hv[j] = og * tanhf(w[j] * cv[j] * rinv);
        ht[j] = hv[j];
      }
    }
    free(pre);
  }
}
