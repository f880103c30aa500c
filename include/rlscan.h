/*
 * rlscan.h -- C ABI of the B200 return-estimation scan library (librlscan.so).
 *
 * Every entry point replaces one launch site of the rl_triton reference
 * (simonsays1980/rl-triton v0.1.3).  The reference binds its kernels from
 * Python through Triton's launcher; this library is bound from Python through
 * ctypes (rl_triton/_native.py), and any other host language can bind the same
 * symbols through ctypes, cffi or a direct C/C++ link.
 *
 * Conventions shared by all entry points
 * --------------------------------------
 *  - All array arguments are DEVICE pointers to row-major, contiguous
 *    [num_envs, seq_len] buffers (row stride == seq_len), 16-byte aligned.
 *    3-D Retrace inputs are [num_envs, seq_len, num_actions].
 *  - `in_dtype` selects the element type of the floating-point input streams
 *    (RLS_F32 or RLS_BF16).  Outputs are always fp32; arithmetic is fp32.
 *    Per-env scalar arrays (last values, seeds, carries, halos) are fp32.
 *  - Flags (terminateds / truncateds / dones) are {0,1} in the input dtype.
 *  - `ws` is a device workspace of at least rls_workspace_bytes(N*T) bytes,
 *    zero-filled ONCE when allocated; the kernels keep it consistent across
 *    calls (an epoch counter lives inside it).  Calls that share one
 *    workspace must be ordered on one stream.
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy stream).
 *  - Before anything is enqueued, every array argument (and the workspace) is
 *    checked to be device (or managed) memory of ONE GPU; anything else (a
 *    host pointer, arrays on two GPUs) returns RLS_ENOTDEVICE.  The call runs
 *    with that GPU current and restores the caller's current device; `stream`
 *    must belong to that GPU.
 *  - Return value: RLS_OK (0) or an RLS_E* status; rls_status_string() names
 *    it.  Launches are asynchronous; device-side failures (a bounded wait that
 *    ran out) are latched in the workspace and read with rls_workspace_error()
 *    (bits: 1 tile look-back, 2 bulk copy, 4 grid barrier).
 */
#ifndef RLSCAN_H
#define RLSCAN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------- */
#define RLS_OK            0
#define RLS_EINVAL        1   /* bad size / enum / null pointer            */
#define RLS_EALIGN        2   /* a pointer is not 16-byte aligned          */
#define RLS_EWORKSPACE    3   /* workspace missing or too small            */
#define RLS_ECUDA         4   /* CUDA launch / runtime error               */
#define RLS_EUNSUPPORTED  5   /* combination not implemented               */
#define RLS_ETOOLARGE     6   /* larger than rls_gae_noalloc's fixed scratch */
#define RLS_ENOTDEVICE    7   /* an array is not device memory of one GPU  */

/* ---- input element types --------------------------------------------- */
#define RLS_F32   0
#define RLS_BF16  1

/* ---- bootstrap kinds (`boot_kind`) -------------------------------------
 * How the optional `bootstrap` argument is read.  The shim picks the kind that
 * reproduces the reference's dispatch exactly (see each op's docstring).   */
#define RLS_BOOT_NONE     0  /* no bootstrap: zero continuation value      */
#define RLS_BOOT_ROW      1  /* fp32 [num_envs]: value at the window end   */
#define RLS_BOOT_LASTCOL  2  /* [num_envs, seq_len], only column T-1 read  */
#define RLS_BOOT_FULL_ADD 3  /* [num_envs, seq_len], additive per step     */
#define RLS_BOOT_FULL_SEL 4  /* [num_envs, seq_len], selected at truncs    */

/* ---- algorithms (for the time-split helpers) --------------------------- */
#define RLS_ALG_GAE         0
#define RLS_ALG_LAMBDA      1
#define RLS_ALG_DISCOUNTED  2
#define RLS_ALG_ELIGIBILITY 3
#define RLS_ALG_PREFIX      4
#define RLS_ALG_SCAN_BWD    5
#define RLS_ALG_SCAN_FWD    6

/* Time-split descriptor.  NULL means "the buffer holds whole rows".  When
 * given, the buffer holds columns [t0, t0+seq_len) of rows of global length
 * total_len; the scan treats the local segment edge as a cut with carry 0
 * (rls_segment_reduce / rls_segment_fixup apply the true carry afterwards).
 * `halo` is fp32 [num_envs]: for backward GAE the value V[t0+seq_len] of the
 * next segment; for the forward scans with an "ends at" boundary the flag
 * done[t0-1] of the previous segment; otherwise unused (may be NULL).     */
typedef struct rls_segment {
    int64_t      t0;
    int64_t      total_len;
    const float* halo;
} rls_segment_t;

/* ---- workspace --------------------------------------------------------- */
/* Bytes of workspace any entry point needs for num_elements = N*T. */
size_t rls_workspace_bytes(int64_t num_elements);
/* Reads (and clears) the device error latch of a workspace; synchronises
 * `stream`.  Returns 0 when no bounded wait ran out, else a bit mask
 * (1 = tile look-back wait, 2 = bulk-copy wait).                          */
int rls_workspace_error(void* ws, void* stream);
const char* rls_status_string(int status);
const char* rls_build_info(void);

/* ---- the seven estimators ---------------------------------------------- */

/* GAE.  Replaces gae_fused_kernel launches at src/rl_triton/ops/gae.py:169-189
 * and the chunked path at src/rl_triton/ops/gae.py:192-215.
 * truncateds may be NULL.  boot_kind in {NONE, ROW, LASTCOL, FULL_ADD, FULL_SEL}. */
int rls_gae(const void* rewards, const void* values, const void* terminateds,
            const void* truncateds, const void* bootstrap, int boot_kind,
            float* advantages, int64_t num_envs, int64_t seq_len,
            float gamma, float lambda_, int in_dtype,
            const rls_segment_t* seg, void* ws, size_t ws_bytes, void* stream);

/* V-trace targets and advantages.  Replaces vtrace_fused_kernel launches at
 * src/rl_triton/ops/vtrace_fused.py:172-218 and the chunked path at
 * src/rl_triton/ops/vtrace.py:161-201.  boot_kind in {NONE, ROW, LASTCOL,
 * FULL_ADD}.  No time split.                                                */
int rls_vtrace(const void* log_pi_target, const void* log_pi_behavior,
               const void* values, const void* rewards, const void* terminateds,
               const void* truncateds, const void* bootstrap, int boot_kind,
               float* targets, float* advantages,
               int64_t num_envs, int64_t seq_len,
               float gamma, float rho_bar, float c_bar, int in_dtype,
               void* ws, size_t ws_bytes, void* stream);

/* Retrace(lambda) targets and advantages (fp32 only; actions int64).
 * Replaces retrace_fused_kernel at src/rl_triton/ops/retrace_fused.py:93-117
 * and the unfused reroute at src/rl_triton/ops/retrace.py:177-196.         */
int rls_retrace(const float* action_probs_target, const float* action_probs_behavior,
                const float* q_values, const float* next_q_values_all,
                const int64_t* actions, const float* rewards,
                const float* terminateds, const float* truncateds,
                float* targets, float* advantages,
                int64_t num_envs, int64_t seq_len, int64_t num_actions,
                float gamma, float lambda_, float c_bar, float rho_bar,
                void* ws, size_t ws_bytes, void* stream);

/* TD(lambda) returns.  Replaces lambda_returns_fused_kernel at
 * src/rl_triton/ops/returns.py:122-147 and the chunked path at :149-152.
 * boot_kind in {NONE, LASTCOL, FULL_ADD}.                                   */
int rls_lambda_returns(const void* rewards, const void* next_values,
                       const void* terminateds, const void* truncateds,
                       const void* bootstrap, int boot_kind, float* out,
                       int64_t num_envs, int64_t seq_len,
                       float gamma, float lambda_, int in_dtype,
                       const rls_segment_t* seg, void* ws, size_t ws_bytes, void* stream);

/* Discounted returns.  Replaces discounted_returns_fused_kernel at
 * src/rl_triton/ops/returns.py:235-259 and the chunked path at :261-263.
 * boot_kind in {NONE, LASTCOL, FULL_ADD}.                                   */
int rls_discounted_returns(const void* rewards, const void* terminateds,
                           const void* truncateds, const void* bootstrap, int boot_kind,
                           float* out, int64_t num_envs, int64_t seq_len,
                           float gamma, int in_dtype,
                           const rls_segment_t* seg, void* ws, size_t ws_bytes, void* stream);

/* Eligibility traces (forward).  Replaces eligibility_traces_fused_kernel at
 * src/rl_triton/ops/returns.py:337-346.  seed_values (fp32 [N]) may be NULL. */
int rls_eligibility_traces(const void* gradients, const void* dones,
                           const float* seed_values, float* out,
                           int64_t num_envs, int64_t seq_len,
                           float gamma, float lambda_, int in_dtype,
                           const rls_segment_t* seg, void* ws, size_t ws_bytes, void* stream);

/* Episodic prefix sum (forward).  Replaces prefix_sum_fused_kernel at
 * src/rl_triton/ops/prefix_sum.py:101-111.  boundary_ends_at: 1 = "ends_at",
 * 0 = "starts_at".  No seq_len limit (the reference asserts <= 131072).     */
int rls_prefix_sum(const void* inputs, const void* dones, const float* seed_values,
                   int boundary_ends_at, float* out,
                   int64_t num_envs, int64_t seq_len, int in_dtype,
                   const rls_segment_t* seg, void* ws, size_t ws_bytes, void* stream);

/* Generic affine scan on precomputed coefficients (fp32):
 *   direction 0 (backward): out[t] = u[t] + v[t]*out[t+1], out[T] = carry
 *   direction 1 (forward):  out[t] = u[t] + v[t]*out[t-1], out[-1] = carry
 * carry (fp32 [N]) may be NULL (zero).  Replaces backward_scan_kernel /
 * chunked_backward_scan_kernel (src/rl_triton/ops/_scan.py:120-142) and
 * forward_scan_kernel (src/rl_triton/ops/_scan.py:203-212).                */
int rls_affine_scan(const float* u, const float* v, const float* carry, int direction,
                    float* out, int64_t num_envs, int64_t seq_len,
                    const rls_segment_t* seg, void* ws, size_t ws_bytes, void* stream);

/* ---- fused epilogues (no counterpart in the reference: its ROADMAP.md lists
 * "fused GAE + advantage normalisation" for v0.2) ------------------------- */

/* GAE with the advantages normalised over the whole batch, as a PPO update
 * uses them:  A = GAE (arguments as rls_gae, no time split),
 *   mean = sum(A) / M,  std = sqrt(sum((A - mean)^2) / (M - 1))  (M = N*T,
 *   unbiased like torch.std),  normalized = (A - mean) / (std + eps).
 * Optional outputs (NULL to skip): returns = A + V (the value targets), the
 * raw advantages A, and stats = fp32[2] {mean, std}.  Two launches: GAE with
 * per-CTA fp64 partial sums (the advantages go to `advantages`, or to
 * `normalized` as scratch), then the normalisation; rows that do not start
 * 16-byte aligned take one more pass.  The workspace (as for rls_gae) holds
 * the partial sums.  Results are deterministic.                               */
int rls_gae_normalized(const void* rewards, const void* values, const void* terminateds,
                       const void* truncateds, const void* bootstrap, int boot_kind,
                       float* normalized, float* returns, float* advantages, float* stats,
                       int64_t num_envs, int64_t seq_len, float gamma, float lambda_, float eps,
                       int in_dtype, void* ws, size_t ws_bytes, void* stream);

/* GAE and the value loss of a PPO update in one pass.  For the value head's
 * predictions V' (fp32 [N, T]):  A = GAE (arguments as rls_gae),
 *   returns = A + V,  d = V' - returns,
 *   loss = mean(d^2)  (RLS_LOSS_MSE, torch.nn.functional.mse_loss)  or
 *          mean(|d| < delta ? d^2 / 2 : delta * (|d| - delta / 2))  (RLS_LOSS_HUBER,
 *          torch.nn.functional.huber_loss),
 * written to loss (fp32 scalar), and its gradient with respect to V' to grad
 * (fp32 [N, T]) for the backward pass.  advantages and returns may be NULL.
 * The per-CTA partial sums live in the workspace; deterministic.             */
#define RLS_LOSS_MSE   0
#define RLS_LOSS_HUBER 1
int rls_gae_value_loss(const void* rewards, const void* values, const void* terminateds,
                       const void* truncateds, const void* bootstrap, int boot_kind,
                       const float* new_values, float* advantages, float* returns, float* grad,
                       float* loss, int64_t num_envs, int64_t seq_len, float gamma, float lambda_,
                       int loss_kind, float delta, int in_dtype, void* ws, size_t ws_bytes, void* stream);

/* GAE with observation-skip masking for multi-turn / tool-use rollouts (the
 * boundary mode the reference's ROADMAP.md lists for v0.2): tokens with
 * mask 0 (observations) pass the recurrence through unchanged, and a
 * generated token's TD error uses the value of the next generated token:
 *   NV[t] = V of the next token after t with mask 1 (0 if none),
 *   A[t]  = mask[t] ? r[t] + gamma*NV[t] - V[t] + gamma*lambda*A[t+1] : A[t+1],
 *   A[T]  = 0.
 * rewards, values and mask are [N, T] in in_dtype (mask in {0, 1});
 * advantages (fp32) is required, returns = A + V (fp32) may be NULL.  One
 * warp per row scans both recurrences chunk by chunk.  No workspace.         */
int rls_gae_obs_skip(const void* rewards, const void* values, const void* mask, float* advantages,
                     float* returns, int64_t num_envs, int64_t seq_len, float gamma, float lambda_,
                     int in_dtype, void* stream);

/* ---- time-split helpers (no counterpart in the reference, which has no
 * multi-GPU support; they implement the carry exchange of a sequence split
 * along time across ranks) ------------------------------------------------ */

/* After the local scan of a segment, summarise each row as the affine map
 * state_at_far_edge = seg_a + seg_b * carry_in_at_near_edge:
 *   backward algorithms: far edge = local column 0, carry enters at column S;
 *   forward algorithms:  far edge = local column S-1, carry enters at column -1.
 * flag0/flag1 are the inputs that determine the decay b[t]:
 *   GAE, LAMBDA, DISCOUNTED: terminateds, truncateds (may be NULL);
 *   ELIGIBILITY, PREFIX: dones, NULL;  SCAN_BWD / SCAN_FWD: v (fp32), NULL.
 * coef: gamma*lambda (GAE, LAMBDA, ELIGIBILITY), gamma (DISCOUNTED), unused
 * otherwise.  flags bit 0: prefix-sum boundary "ends_at".                  */
int rls_segment_reduce(int alg, const void* flag0, const void* flag1, int in_dtype,
                       const float* out, float* seg_a, float* seg_b,
                       int64_t num_envs, int64_t seq_len, float coef, int flags,
                       const rls_segment_t* seg, void* stream);

/* Apply the true incoming carry (fp32 [N]) of each row to a segment's local
 * result: out[t] += P[t] * carry, P[t] = product of b over [t, edge].  Stops
 * at the first zero of P, so the work is bounded by the distance to the first
 * episode reset (or to underflow of the decay product).
 * With flags & RLS_SEG_EXCLUSIVE the carry is the correction entering at the
 * segment's entry element itself, as rls_segment_compose returns it: for
 * backward algorithms P leaves out the entry element's own decay
 * (P[last] = 1), and a NULL halo reads as 0.                                */
#define RLS_SEG_EXCLUSIVE 2
int rls_segment_fixup(int alg, const void* flag0, const void* flag1, int in_dtype,
                      float* out, const float* carry,
                      int64_t num_envs, int64_t seq_len, float coef, int flags,
                      const rls_segment_t* seg, void* stream);

/* One-exchange time split.  Each rank scans its segment with the cut as
 * carry 0 and a zero halo (no value from a neighbour is needed before the
 * scan), then summarises every row in summary[5][N] (fp32):
 *   0: A, the local state at the far edge (column 0 backward, S-1 forward);
 *   1: B, the decay product from the entry element to the far edge (backward:
 *      without the entry element's own decay);
 *   2: backward: alpha, the weight the next segment's first value V carries in
 *      the entry element (GAE: gamma*(1-term[S-1]) where trunc[S-1] == 0, else
 *      0); forward: m, the next segment's entry gate taken from this segment's
 *      last flag (1 - done[S-1] when the gate reads done[t-1], else 1);
 *   3: backward: beta, the entry element's own decay b[S-1]; forward: 0;
 *   4: backward GAE: V[0] of this segment; else 0.
 * `values` is read by GAE only (may be NULL otherwise); gamma is GAE's
 * discount; coef and flags as for rls_segment_reduce.  The ranks all-gather
 * their summaries (20 bytes per row per rank, one collective), and
 * rls_segment_compose turns the W summaries ([W][5][N], rank order) into the
 * correction entering `rank`'s segment, which rls_segment_fixup applies with
 * RLS_SEG_EXCLUSIVE.                                                         */
int rls_segment_summary(int alg, const void* flag0, const void* flag1, const void* values, int in_dtype,
                        const float* out, float* summary, int64_t num_envs, int64_t seq_len, float gamma,
                        float coef, int flags, const rls_segment_t* seg, void* stream);
int rls_segment_compose(const float* summaries, int rank, int world, int backward, int64_t num_envs,
                        float* carry, void* stream);

/* ---- GAE for callers that cannot allocate --------------------------------
 * No counterpart in the reference (its Triton path always allocates through
 * PyTorch).  Same arguments and results as rls_gae, minus the workspace: the
 * look-back scratch lives in a fixed array inside the library
 * (RLS_NOALLOC_MAX_ELEMENTS elements' worth, about 6 MB, held on every GPU
 * that loads the library until the process exits).  Meant for callers that
 * must not call cudaMalloc -- code running while a CUDA graph is being
 * captured into a pool they do not own, real-time loops with a frozen memory
 * budget, or hosts that only hand out buffers they allocated themselves.
 *  - num_envs * seq_len above RLS_NOALLOC_MAX_ELEMENTS returns RLS_ETOOLARGE.
 *  - The call allocates nothing; it clears the scratch's counters with one
 *    small cudaMemsetAsync on `stream`, then launches the same kernels as
 *    rls_gae.  Bounded device waits that run out latch an error bit in the
 *    scratch; rls_gae_noalloc_error() reads it.
 *  - The first call on a device looks the array's device address up
 *    (cudaGetSymbolAddress); make that first call before any stream capture.
 *  - Every call shares the one array: calls that may overlap on the GPU (on
 *    different streams without ordering between them) race and give wrong
 *    results.  Order them on one stream, or use rls_gae with a workspace per
 *    stream.                                                                */
#define RLS_NOALLOC_MAX_ELEMENTS (1LL << 27)
int rls_gae_noalloc(const void* rewards, const void* values, const void* terminateds,
                    const void* truncateds, const void* bootstrap, int boot_kind,
                    float* advantages, int64_t num_envs, int64_t seq_len,
                    float gamma, float lambda_, int in_dtype,
                    const rls_segment_t* seg, void* stream);

/* Error latch of the current device's fixed scratch: synchronises `stream`,
 * returns 0 when no bounded device wait of rls_gae_noalloc ran out since the
 * last read (else the bit mask of rls_workspace_error, or -1 if the scratch
 * cannot be reached) and clears it.  A wait that ran out means that call's
 * advantages are wrong.                                                      */
int rls_gae_noalloc_error(void* stream);

#ifdef __cplusplus
}
#endif
#endif /* RLSCAN_H */
