/*
 * rlscan_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the reference's sequential estimators
 * (simonsays1980/rl-triton v0.1.3), used as the parity checker by tests/,
 * by __graft_entry__.smoke() and as the timed CPU baseline of bench.py.  The
 * product path (rl_triton -> librlscan.so) never calls this file.
 *
 * Compiled twice: REAL=float (suffix _f32, matches the reference's fp32
 * sequential loops) and REAL=double (suffix _f64, a higher-precision
 * yardstick).  Inputs are float arrays, row-major [N, T] ([N, T, A] for the
 * Retrace action tensors); outputs are REAL arrays.  Rows are independent;
 * oracle.py runs row blocks on a thread pool (ctypes releases the GIL).
 *
 * Pinned against the reference's own sequential loops (imported from
 * tests/test_*.py of the reference) by tests/golden/make_golden.py, which
 * writes the golden fixtures checked in tests/test_oracle.py.
 *
 * Bootstrap kinds mirror include/rlscan.h:
 *   0 none, 1 per-row [N], 2 last column of [N,T], 3 full additive, 4 full select.
 * Compile with -ffp-contract=off so the float variant rounds like
 * element-wise PyTorch on the CPU.
 */
#include <math.h>
#include <stdint.h>

#ifndef REAL
#define REAL float
#endif
#ifndef SFX
#define SFX _f32
#endif
#define CAT_(a, b) a##b
#define CAT(a, b) CAT_(a, b)
#define FN(name) CAT(name, SFX)

static inline REAL minr(REAL a, REAL b) { return a < b ? a : b; }

/* Window-end next-state value for GAE / V-trace. */
static inline REAL window_boot(int kind, const float* boot, const float* boot_row, int64_t n, int64_t T) {
    if (kind == 0) return 0;
    if (kind == 1) return (REAL)boot_row[n];
    return (REAL)boot[n * T + T - 1];
}

/*
 * GAE.  Follows tests/test_gae.py:34-60 (reference_gae) and :418-450
 * (_ref_gae_sequential) and the chunked form of src/rl_triton/ops/gae.py:192-215.
 * kind 4 (select): v_next = bootstrap[t] at truncated steps;
 * kind 3 (additive): v_next = values[t+1]*(1-trunc) + bootstrap[t];
 * kinds 0-2 without truncations: v_next = values[t+1].
 */
void FN(orc_gae)(const float* r, const float* v, const float* term, const float* trunc, const float* boot,
                 int kind, REAL* out, int64_t N, int64_t T, double gamma_, double lam_) {
    const REAL gamma = (REAL)(float)gamma_, gl = (REAL)((float)gamma_ * (float)lam_);
    for (int64_t n = 0; n < N; ++n) {
        REAL carry = 0;
        for (int64_t t = T - 1; t >= 0; --t) {
            const int64_t i = n * T + t;
            const REAL tm = term[i], tr = trunc ? trunc[i] : 0;
            const REAL done = trunc ? minr(tm + tr, (REAL)1) : tm;
            REAL vn;
            if (t == T - 1) {
                vn = window_boot(kind == 1 ? 1 : (kind == 0 ? 0 : 2), boot, boot, n, T);
            } else if (kind == 4) {
                vn = (tr == 1) ? (REAL)boot[i] : (REAL)v[i + 1];
            } else {
                vn = trunc ? ((tr == 0) ? (REAL)v[i + 1] : 0) : (REAL)v[i + 1];
                if (kind == 3) vn = vn + (REAL)boot[i];
            }
            const REAL delta = (REAL)r[i] + gamma * vn * (1 - tm) - (REAL)v[i];
            carry = delta + gl * (1 - done) * carry;
            out[i] = carry;
        }
    }
}

/*
 * V-trace.  Follows tests/test_vtrace.py:56-101 (reference_vtrace) and
 * :424-480 (_ref_vtrace_sequential); chunked form src/rl_triton/ops/vtrace.py:161-201.
 */
void FN(orc_vtrace)(const float* lpt, const float* lpb, const float* v, const float* r, const float* term,
                    const float* trunc, const float* boot, int kind, REAL* vs, REAL* adv, int64_t N, int64_t T,
                    double gamma_, double rho_bar_, double c_bar_) {
    const REAL gamma = (REAL)(float)gamma_, rho_bar = (REAL)(float)rho_bar_, c_bar = (REAL)(float)c_bar_;
    for (int64_t n = 0; n < N; ++n) {
        REAL carry = 0;
        for (int64_t t = T - 1; t >= 0; --t) {
            const int64_t i = n * T + t;
            const REAL ratio = (REAL)exp((double)((REAL)lpt[i] - (REAL)lpb[i]));
            const REAL rho = minr(ratio, rho_bar), c = minr(ratio, c_bar);
            const REAL tm = term[i], tr = trunc ? trunc[i] : 0;
            const REAL done = trunc ? minr(tm + tr, (REAL)1) : tm;
            REAL vn;
            if (t == T - 1) {
                vn = window_boot(kind, boot, boot, n, T);
            } else {
                vn = trunc ? ((tr == 0) ? (REAL)v[i + 1] : 0) : (REAL)v[i + 1];
                if (kind == 3) vn = vn + (REAL)boot[i];
            }
            const REAL delta = rho * ((REAL)r[i] + gamma * vn * (1 - tm) - (REAL)v[i]);
            carry = delta + gamma * c * (1 - done) * carry;
            vs[i] = carry + (REAL)v[i];
        }
        for (int64_t t = 0; t < T; ++t) {
            const int64_t i = n * T + t;
            const REAL ratio = (REAL)exp((double)((REAL)lpt[i] - (REAL)lpb[i]));
            const REAL rho = minr(ratio, rho_bar);
            const REAL tm = term[i], tr = trunc ? trunc[i] : 0;
            REAL vsn;
            if (t == T - 1) {
                vsn = window_boot(kind, boot, boot, n, T);
            } else {
                vsn = trunc ? ((tr == 0) ? vs[i + 1] : 0) : vs[i + 1];
                if (kind == 3) vsn = vsn + (REAL)boot[i];
            }
            adv[i] = rho * ((REAL)r[i] + gamma * vsn * (1 - tm) - (REAL)v[i]);
        }
    }
}

/*
 * Retrace(lambda).  Follows tests/test_retrace.py:19-60 (reference_retrace).
 * Actions outside [0, A) select probability 0 (the fused kernel's one-hot
 * gather, src/rl_triton/kernels/retrace_fused.py:155-158).
 */
void FN(orc_retrace)(const float* pi, const float* mu, const float* q, const float* nq, const int64_t* act,
                     const float* r, const float* term, const float* trunc, REAL* qret, REAL* adv, int64_t N,
                     int64_t T, int64_t A, double gamma_, double lam_, double c_bar_, double rho_bar_) {
    const REAL gamma = (REAL)(float)gamma_, lam = (REAL)(float)lam_;
    const REAL c_bar = (REAL)(float)c_bar_, rho_bar = (REAL)(float)rho_bar_;
    for (int64_t n = 0; n < N; ++n) {
        REAL carry = 0;
        REAL c_next = 0; /* c[T] = 0 */
        for (int64_t t = T - 1; t >= 0; --t) {
            const int64_t i = n * T + t;
            REAL e = 0;
            for (int64_t a = 0; a < A; ++a) e += (REAL)pi[i * A + a] * (REAL)nq[i * A + a];
            const int64_t a_t = act[i];
            const REAL pa = (a_t >= 0 && a_t < A) ? (REAL)pi[i * A + a_t] : 0;
            const REAL ratio = pa / (REAL)mu[i];
            const REAL tm = term[i], done = minr(tm + (REAL)trunc[i], (REAL)1);
            const REAL delta = (REAL)r[i] + gamma * e * (1 - tm) - (REAL)q[i];
            carry = delta + gamma * c_next * (1 - done) * carry;
            qret[i] = carry + (REAL)q[i];
            c_next = lam * minr(ratio, c_bar);
        }
        for (int64_t t = 0; t < T; ++t) {
            const int64_t i = n * T + t;
            const int64_t a_t = act[i];
            const REAL pa = (a_t >= 0 && a_t < A) ? (REAL)pi[i * A + a_t] : 0;
            const REAL rho = minr(pa / (REAL)mu[i], rho_bar);
            const REAL qn = (t + 1 < T) ? qret[i + 1] : 0;
            adv[i] = rho * ((REAL)r[i] + gamma * qn * (1 - (REAL)term[i]) - (REAL)q[i]);
        }
    }
}

/*
 * TD(lambda) returns.  Follows tests/test_returns.py:19-39
 * (reference_lambda_returns) and :451-483 (_ref_lambda_sequential).
 * kind 0: no bootstrap; 2: carry = bootstrap[:, -1]; 3: also gamma*trunc*boot in u.
 */
void FN(orc_lambda)(const float* r, const float* nv, const float* term, const float* trunc, const float* boot,
                    int kind, REAL* out, int64_t N, int64_t T, double gamma_, double lam_) {
    const REAL gamma = (REAL)(float)gamma_, lam = (REAL)(float)lam_;
    for (int64_t n = 0; n < N; ++n) {
        REAL carry = (kind >= 2) ? (REAL)boot[n * T + T - 1] : 0;
        for (int64_t t = T - 1; t >= 0; --t) {
            const int64_t i = n * T + t;
            const REAL tr = trunc ? trunc[i] : 0;
            const REAL done = trunc ? minr((REAL)term[i] + tr, (REAL)1) : (REAL)term[i];
            const REAL nd = 1 - done;
            REAL g = (REAL)r[i] + gamma * (1 - lam) * nd * (REAL)nv[i] + gamma * lam * nd * carry;
            if (kind == 3) g = g + gamma * tr * (REAL)boot[i];
            carry = g;
            out[i] = carry;
        }
    }
}

/*
 * Discounted returns.  Follows tests/test_returns.py:42-57
 * (reference_discounted_returns) and :486-511 (_ref_discounted_sequential).
 */
void FN(orc_discounted)(const float* r, const float* term, const float* trunc, const float* boot, int kind,
                        REAL* out, int64_t N, int64_t T, double gamma_) {
    const REAL gamma = (REAL)(float)gamma_;
    for (int64_t n = 0; n < N; ++n) {
        REAL carry = (kind >= 2) ? (REAL)boot[n * T + T - 1] : 0;
        for (int64_t t = T - 1; t >= 0; --t) {
            const int64_t i = n * T + t;
            const REAL tr = trunc ? trunc[i] : 0;
            const REAL done = trunc ? minr((REAL)term[i] + tr, (REAL)1) : (REAL)term[i];
            REAL g = (REAL)r[i] + gamma * (1 - done) * carry;
            if (kind == 3) g = g + gamma * tr * (REAL)boot[i];
            carry = g;
            out[i] = carry;
        }
    }
}

/*
 * Eligibility traces (forward).  Follows tests/test_returns.py:362-385
 * (reference_eligibility_traces).
 */
void FN(orc_eligibility)(const float* g, const float* dones, const float* seed, REAL* out, int64_t N, int64_t T,
                         double gamma_, double lam_) {
    const REAL gl = (REAL)((float)gamma_ * (float)lam_);
    for (int64_t n = 0; n < N; ++n) {
        REAL carry = seed ? (REAL)seed[n] : 0;
        REAL prev = 0;
        for (int64_t t = 0; t < T; ++t) {
            const int64_t i = n * T + t;
            carry = (REAL)g[i] + gl * (1 - prev) * carry;
            out[i] = carry;
            prev = dones[i];
        }
    }
}

/*
 * Episodic prefix sum (forward).  Follows tests/test_prefix_sum.py:18-58
 * (reference_episodic_prefix_sum); ends_at = 1 gates on done[t-1].
 */
void FN(orc_prefix)(const float* x, const float* dones, const float* seed, int ends_at, REAL* out, int64_t N,
                    int64_t T) {
    for (int64_t n = 0; n < N; ++n) {
        REAL carry = seed ? (REAL)seed[n] : 0;
        REAL prev = 0;
        for (int64_t t = 0; t < T; ++t) {
            const int64_t i = n * T + t;
            const REAL flag = ends_at ? prev : (REAL)dones[i];
            carry = (REAL)x[i] + (1 - flag) * carry;
            out[i] = carry;
            prev = dones[i];
        }
    }
}

/*
 * Generic scans.  Follows tests/test_scan_chunked.py:15-29 (_reference_scan)
 * for the backward direction; the forward direction is its mirror
 * (src/rl_triton/kernels/scan.py:91-138).
 */
void FN(orc_scan)(const float* u, const float* v, const float* carry0, int direction, REAL* out, int64_t N,
                  int64_t T) {
    for (int64_t n = 0; n < N; ++n) {
        REAL carry = carry0 ? (REAL)carry0[n] : 0;
        for (int64_t k = 0; k < T; ++k) {
            const int64_t t = direction == 0 ? (T - 1 - k) : k;
            const int64_t i = n * T + t;
            carry = (REAL)u[i] + (REAL)v[i] * carry;
            out[i] = carry;
        }
    }
}

/*
 * GAE with observation-skip masking.  No code counterpart in the reference:
 * restates the boundary mode its ROADMAP.md (v0.2, "Multi-turn /
 * observation-skip masking") describes -- masked tokens pass the recurrence
 * through unchanged and the next valid token's TD error uses the pre-skip
 * value.  Sequential loop: nextvalue and the running advantage are carried
 * backward and only updated at tokens with mask 1.
 */
void FN(orc_gae_obs_skip)(const float* r, const float* v, const float* mask, REAL* adv, REAL* ret, int64_t N,
                          int64_t T, double gamma_, double lam_) {
    const REAL gamma = (REAL)(float)gamma_, gl = (REAL)((float)gamma_ * (float)lam_);
    for (int64_t n = 0; n < N; ++n) {
        REAL nextvalue = 0, running = 0;
        for (int64_t t = T - 1; t >= 0; --t) {
            const int64_t i = n * T + t;
            if (mask[i] != 0) {
                const REAL delta = (REAL)r[i] + gamma * nextvalue - (REAL)v[i];
                running = delta + gl * running;
                nextvalue = (REAL)v[i];
            }
            adv[i] = running;
            ret[i] = running + (REAL)v[i];
        }
    }
}
