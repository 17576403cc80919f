/*
 * gsdft_b200.h — C ABI of the B200-native screened density-fitted Coulomb (RI-J) path.
 *
 * Replaces the JAX hot path of andresguzco/gs-dft: the significant-pair list, the product auxiliary
 * basis with its Coulomb metric and Cholesky factor, the fused 3-centre (aux | splat-pair) fit-vector
 * contraction gamma, the metric solve, and the analytic backward pass to the splat chart parameters.
 *
 * Conventions (every entry point):
 *   - all pointers are DEVICE pointers unless the name ends in _host; FP64 arrays are row-major;
 *   - buffers are owned and allocated by the caller, and scratch comes from an explicit workspace
 *     whose size the matching *_workspace_size() returns. No entry point allocates device memory for
 *     its data, and no entry point calls a math library (cuBLAS, cuSOLVER): the dense contractions
 *     and factorisations are the library's own DMMA kernels;
 *   - work is enqueued on `stream` (the last argument). Only gsdft_pairs_count / gsdft_pairs_build /
 *     gsdft_pair_plan / gsdft_aux_cholesky synchronise the stream, to read back integers (pair counts,
 *     the factorisation status), exactly where the reference syncs to the host
 *     (gs_dft/screening/pairs.py:279,305);
 *   - the return value is a status: 0 = GSDFT_OK, otherwise an error code; gsdft_last_error_string()
 *     describes the last failure on the calling thread;
 *   - outputs are deterministic: identical inputs give bit-identical outputs (no floating-point
 *     atomics; every reduction has a fixed order).
 *
 * Layouts:
 *   quat (M,4), log_scale (M,3), centers (M,3)           splat chart parameters
 *   A9 (M,9) row-major 3x3 precision, N (M)              splat quantities
 *   pi, pj int32 (n), w double (n)                       pair list; w = 0/1 (ordered) or 0/1/2 (unique)
 *   beta (Naux), R (Naux,3), KN (Naux)                   isotropic aux: exponent, centre, normalisation
 *   V / L (Naux,Naux)                                     metric; L = lower Cholesky factor, row-major
 *   C_occ (M,n_occ), occ (n_occ)                         occupied orbitals and occupations
 *   gA6 (M,6)                                             symmetric cotangent [xx,yy,zz,xy,xz,yz]
 */
#ifndef GSDFT_B200_H
#define GSDFT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* gsdft_stream_t; /* = cudaStream_t */

enum {
  GSDFT_OK = 0,
  GSDFT_ERR_ARG = 1,       /* bad shape, size, pointer or workspace */
  GSDFT_ERR_CUDA = 2,      /* a CUDA runtime call or launch failed */
  GSDFT_ERR_OVERFLOW = 3,  /* more significant pairs than the headroom allows */
  GSDFT_ERR_LINALG = 4     /* the metric is not positive definite, or a library call failed */
};

/* Fields of one live pair's record, stored record-major: rec[a * GSDFT_REC_FIELDS + f]
 * (144 bytes per pair, so any tile of records is a 16-byte-aligned contiguous block). */
enum {
  GSDFT_REC_L0 = 0, GSDFT_REC_L1, GSDFT_REC_L2,                     /* eigenvalues of A_hat */
  GSDFT_REC_U00, GSDFT_REC_U01, GSDFT_REC_U02,                      /* eigenvectors (columns) */
  GSDFT_REC_U10, GSDFT_REC_U11, GSDFT_REC_U12,
  GSDFT_REC_U20, GSDFT_REC_U21, GSDFT_REC_U22,
  GSDFT_REC_P0, GSDFT_REC_P1, GSDFT_REC_P2,                         /* product centre */
  GSDFT_REC_QK,                                                     /* q * KN * pref */
  GSDFT_REC_Q,                                                      /* q = w sum occ C_i C_j */
  GSDFT_REC_KN,                                                     /* KN * pref */
  GSDFT_REC_FIELDS
};

/* Per-live-pair sums of the reverse pass, stored record-major: sums[a * GSDFT_VJP_FIELDS + f]. */
enum {
  GSDFT_VJP_SJ = 0,
  GSDFT_VJP_SD0, GSDFT_VJP_SD1, GSDFT_VJP_SD2,
  GSDFT_VJP_SV0, GSDFT_VJP_SV1, GSDFT_VJP_SV2,
  GSDFT_VJP_SZ00, GSDFT_VJP_SZ11, GSDFT_VJP_SZ22, GSDFT_VJP_SZ01, GSDFT_VJP_SZ02, GSDFT_VJP_SZ12,
  GSDFT_VJP_FIELDS
};

#define GSDFT_SIDE_FIELDS 20 /* per live pair: i-side (gA6, gmu3, gN) then j-side */

/* Per-representative cotangents handed to gsdft_pair_chain directly (xc[a * GSDFT_XC_FIELDS + f]):
 * of A_hat (the symmetric matrix's entries), of P, of KN (the product N_i N_j exp(...)), and dE/dq
 * per unit weight. Written by gsdft_exact_j_vjp. */
enum {
  GSDFT_XC_A00 = 0, GSDFT_XC_A11, GSDFT_XC_A22, GSDFT_XC_A01, GSDFT_XC_A02, GSDFT_XC_A12,
  GSDFT_XC_P0, GSDFT_XC_P1, GSDFT_XC_P2,
  GSDFT_XC_KN,
  GSDFT_XC_J,
  GSDFT_XC_FIELDS
};

/* Version of this ABI (entry points, argument meaning, record layouts); gsdft_version() returns it.
 * A host binding checks it at load time so that a library built from older sources is refused. */
#define GSDFT_ABI_VERSION 4

const char* gsdft_last_error_string(void);
int gsdft_version(void);

/* Reads (and with clear != 0 resets) the library's device status word on the current device:
 * nonzero when a kernel's bounded wait on a bulk copy ran out (the kernel then abandoned its work
 * and its outputs are invalid). Synchronises the device. No reference counterpart. */
int gsdft_device_status(int* status_host, int clear);

/* Cumulative number of kernels this library has launched in the process (all devices). Used to
 * report how many of the library's own kernels ran in a timed region. No reference counterpart. */
int64_t gsdft_kernel_launches(void);

/* FP64 FMA throughput probe: blocks x threads threads each run 16 independent FMA chains for
 * `iters` iterations (2 * 16 * iters flop per thread) and write one sum per thread to out
 * (blocks * threads doubles). Measures the device's FP64 peak at the clocks of the run. No
 * reference counterpart. */
int gsdft_dfma_probe(double* out, int64_t iters, int blocks, int threads, gsdft_stream_t stream);

/* Node screening of the integral kernels' 20-node Laplace sums (gsdft_j_forward, its no-allocation
 * variant, gsdft_j_vjp, gsdft_j_vjp_weighted): along the nodes the exponent of an (aux, pair) term
 * never decreases and its prefactor never increases, so once a warp's every term has an exponent
 * 2^-87 below its first node's, the remaining nodes are below the last bit of the sums and the warp
 * stops. On by default; enabled = 0 evaluates all 20 nodes everywhere (the reference's sum, term by
 * term). A process-wide setting read at each launch (a CUDA graph keeps the value it was captured
 * with). No reference counterpart: the reference always sums 20 nodes (gs_dft/coulomb/ri.py:175-185). */
int gsdft_set_node_screening(int enabled);
int gsdft_node_screening(void);

/* Node evaluations ((aux, pair) units times the nodes each evaluated, 20 without screening) of the
 * forward and reverse integral kernels on the current device since the last clear; clear != 0 resets
 * them. Synchronises the device. For work accounting (the roofline's evaluated FLOP count). No
 * reference counterpart. */
int gsdft_node_evals(uint64_t* forward_host, uint64_t* reverse_host, int clear);

/* C = alpha op(A) op(B) + beta C on the FP64 tensor cores (mma.sync f64), row-major, op = transpose
 * when trans_a / trans_b (A then stored K x M, B stored N x K); M, N, K >= 0, leading dimensions in
 * elements. The GEMM under the library's Cholesky, factor inverse and RI-K contractions, exported
 * for direct use and testing. No reference counterpart (the reference's dense algebra is XLA's). */
int gsdft_dense_gemm(int trans_a, int trans_b, int64_t M, int64_t N, int64_t K, double alpha,
                     const double* A, int64_t lda, const double* B, int64_t ldb, double beta,
                     double* C, int64_t ldc, gsdft_stream_t stream);

/* ---- splat chart ------------------------------------------------------------------------------ */

/* A = R(q) diag(exp l) R(q)^T, N = (8 exp(sum l) / pi^3)^(1/4).
 * Replaces Splat.A / Splat.norm / full_quantities (gs_dft/basis/spectral.py:33-40,71-82;
 * gs_dft/coulomb/stream.py:79-81). */
int gsdft_splat_quantities(const double* quat, const double* log_scale, int64_t M, double* A9,
                           double* N, gsdft_stream_t stream);

/* Reverse of the chart: (gA6, gN) -> (g_quat, g_log_scale). The jax.grad of the same chart
 * (gs_dft/basis/spectral.py:33-40,71-82), written out. */
int gsdft_chart_vjp(const double* quat, const double* log_scale, const double* gA6,
                    const double* gN, int64_t M, double* g_quat, double* g_log_scale,
                    gsdft_stream_t stream);

/* ---- significant-pair list ------------------------------------------------------------------- */

size_t gsdft_pairs_workspace_size(int64_t M, int64_t pad_to);

/* Number of pairs with |S_ij| > eps (j >= i when unique). Replaces _count_significant
 * (gs_dft/screening/pairs.py:103-118). Synchronises the stream. */
int gsdft_pairs_count(const double* A9, const double* mu, const double* N, int64_t M, double eps,
                      int unique, int64_t* n_sig_host, void* ws, size_t ws_bytes,
                      gsdft_stream_t stream);

/* The lexsorted significant list padded to pad_to with (0,0,w=0); if more than pad_to pairs are
 * significant, keeps the pad_to largest |S| (ties by ascending flat index), re-lexsorted; fails
 * with GSDFT_ERR_OVERFLOW above 2*pad_to. eps < 0 keeps every pair. Replaces neighbor_pairs with
 * pad_to (gs_dft/screening/pairs.py:225-315, 155-164, 318-322). Synchronises the stream. */
int gsdft_pairs_build(const double* A9, const double* mu, const double* N, int64_t M, double eps,
                      int unique, int64_t pad_to, int32_t* pi, int32_t* pj, double* w,
                      int64_t* n_sig_host, void* ws, size_t ws_bytes, gsdft_stream_t stream);

/* Round-robin deal of a padded list over G devices, new[g*d + j] = old[j*G + g]; identity when
 * G <= 1 or n % G != 0. Replaces stripe_pairs (gs_dft/ks/shard.py:146-166). */
int gsdft_stripe_pairs(const int32_t* pi, const int32_t* pj, const double* w, int64_t n, int G,
                       int32_t* pi_out, int32_t* pj_out, double* w_out, gsdft_stream_t stream);

/* Refresh-time plan of a pair list, step 1 — representatives: the live entries (w != 0) in list
 * order, where with merge_twins != 0 a live (i,j), i < j, whose transpose (j,i) is also live (each
 * occurring once) represents both: the two carry the same 3-centre integral, so the pair is
 * evaluated once with the summed weight, and J is written to both list positions. rep_pos (list
 * position), rep_w (summed weight), rep_twin (list position of the merged transpose or -1), each
 * n_rep long (at most the live count). Synchronises the stream (returns n_rep). The identity is the
 * one behind the reference's unique-pair mode (gs_dft/screening/pairs.py:229-233; its test
 * tests/unit/test_pair_tricks.py:81-100); the reference evaluates both orientations. */
size_t gsdft_pair_plan_workspace_size(int64_t n, int64_t M);
int gsdft_pair_reps(const int32_t* pi, const int32_t* pj, const double* w, int64_t n, int64_t M,
                    int merge_twins, int32_t* rep_pos, double* rep_w, int32_t* rep_twin,
                    int64_t* n_rep_host, void* ws, size_t ws_bytes, gsdft_stream_t stream);

/* Step 2 — groupings of a contiguous slice of representatives (all of them on one device, one
 * rank's share on several): order_i / order_j (n_rep) list the slice's representatives stably
 * sorted by pi / pj, seg_i / seg_j (M+1) are the segment offsets, partner_i / partner_j (n_rep)
 * the other splat of each sorted entry (pj of the by-pi grouping, pi of the by-pj one). Used by
 * the deterministic per-splat reductions (the reference scatters with segment sums inside
 * autodiff). */
size_t gsdft_pair_groups_workspace_size(int64_t n_rep, int64_t M);
int gsdft_pair_groups(const int32_t* pi, const int32_t* pj, const int32_t* rep_pos, int64_t n_rep,
                      int64_t M, int32_t* order_i, int64_t* seg_i, int32_t* partner_i,
                      int32_t* order_j, int64_t* seg_j, int32_t* partner_j, void* ws,
                      size_t ws_bytes, gsdft_stream_t stream);

/* Estimated integral cost of each representative (int64, n_rep), for partitioning the list across
 * devices by work: over every (n_aux / n_sample)-th aux, the number of Laplace nodes the integral
 * kernels' node screening would evaluate for that (aux, pair), plus one for the fixed per-(aux, pair)
 * work. Integer costs make the prefix sums that cut the list exact, so every rank computes the same
 * cut. Refresh-time. The north star's "balanced by estimated integral cost"; the reference deals
 * the padded list round-robin instead (gs_dft/ks/shard.py:146-166). */
int gsdft_rep_cost(const double* A9, const double* mu, int64_t M, const int32_t* pi,
                   const int32_t* pj, const int32_t* rep_pos, int64_t n_rep, const double* beta,
                   const double* R, int64_t n_aux, int64_t n_sample, int64_t* cost,
                   gsdft_stream_t stream);

/* ---- auxiliary basis, metric, factor ------------------------------------------------------------ */

/* Frozen product aux: per listed pair (pi == NULL: the M self-products), alpha0 = det(A_hat)^(1/3)
 * (1 on zero-weight entries), centre = product centre; log_alpha = log(alpha0 * s) for each scale s,
 * scale-major (Naux = n * n_scales). Replaces init_product_aux (gs_dft/basis/isotropic.py:81-116). */
int gsdft_product_aux(const double* A9, const double* mu, const double* N, int64_t M,
                      const int32_t* pi, const int32_t* pj, const double* w, int64_t n_pairs,
                      const double* scales_host, int n_scales, double* log_alpha, double* R,
                      gsdft_stream_t stream);

/* beta = exp(log_alpha), KN = (2 beta / pi)^(3/4). Replaces IsotropicSplat.alpha/.norm and
 * aux_quantities (gs_dft/basis/isotropic.py:30-39; gs_dft/coulomb/ri.py:238-240). */
int gsdft_aux_quantities(const double* log_alpha, int64_t n_aux, double* beta, double* KN,
                         gsdft_stream_t stream);

/* V_PQ = KN_P KN_Q 2 pi^2.5 / (b_P b_Q sqrt(b_P + b_Q)) F0(b_P b_Q/(b_P+b_Q) |R_P - R_Q|^2),
 * F0 from erf. Replaces aux_metric / coulomb_block (gs_dft/coulomb/ri.py:63-123,267-275). */
int gsdft_aux_metric(const double* beta, const double* R, const double* KN, int64_t n_aux,
                     double* V, gsdft_stream_t stream);

/* In place: V <- lower Cholesky factor of V + lam I (row-major; the strict upper triangle is
 * zeroed). Replaces aux_cholesky / shift_diag / _chol_donated (gs_dft/coulomb/ri.py:243-264).
 * Fails with GSDFT_ERR_LINALG if V + lam I is not positive definite. Synchronises the stream. */
size_t gsdft_aux_cholesky_workspace_size(int64_t n_aux);
int gsdft_aux_cholesky(double* V, int64_t n_aux, double lam, void* ws, size_t ws_bytes,
                       gsdft_stream_t stream);

/* ---- per-step J-build ---------------------------------------------------------------------------- */

/* Per pair representative: A_hat, P, KN (gs_dft/coulomb/stream.py:203-215), the eigen-decomposition of A_hat
 * (gs_dft/coulomb/ri.py:145), and q = w sum_o occ_o C_io C_jo (gs_dft/coulomb/ri.py:456), for
 * each representative (w its summed weight). With n_occ = 0 and C_occ = NULL, Q and QK are left
 * unwritten, for gsdft_block_density to fill (n_occ = 0 with C_occ set writes q = 0).
 * rec is (n_rep, GSDFT_REC_FIELDS). */
int gsdft_pair_prep(const double* A9, const double* mu, const double* N, int64_t M,
                    const int32_t* pi, const int32_t* pj, const int32_t* rep_pos,
                    const double* rep_w, int64_t n_rep, const double* C_occ, const double* occ,
                    int64_t n_occ, double* rec, gsdft_stream_t stream);

/* gamma_P = sum_a (P|a) q_a over the pair representatives, the 3-centre integral fused with the contraction
 * (never stored). Replaces df_coulomb_gamma_screened + full_isobra_block
 * (gs_dft/coulomb/ri.py:436-469, 126-185). */
size_t gsdft_j_forward_workspace_size(int64_t n_rep, int64_t n_aux);
int gsdft_j_forward(const double* rec, int64_t n_rep, const double* beta, const double* R,
                    const double* KN, int64_t n_aux, double* gamma, void* ws, size_t ws_bytes,
                    gsdft_stream_t stream);

/* gsdft_j_forward without a workspace and without allocating: for callers that cannot allocate
 * device memory at call time and cannot pass a workspace — for instance a handler inside a framework
 * that owns the device memory pool (XLA preallocates most of the GPU for its own allocator, so a
 * cudaMalloc from a custom call can fail or fragment that pool), or code with a fixed memory budget.
 * The per-split partial sums live in one fixed device array of 2^20 doubles (8 MiB) that every GPU
 * loading the library holds until the process exits; n_aux above 2^20 is rejected (GSDFT_ERR_ARG).
 * The first call on each device looks up that array's device address (cudaGetSymbolAddress), so
 * make the first call on a device before any stream capture. All calls share the array and it keeps
 * the last call's contents (nothing in it needs to start at zero): calls whose work overlaps on the
 * GPU — concurrent streams, or several host threads on one device — race on it and must be
 * serialised by the caller. No counterpart in the reference. */
int gsdft_j_forward_noalloc(const double* rec, int64_t n_rep, const double* beta, const double* R,
                            const double* KN, int64_t n_aux, double* gamma, gsdft_stream_t stream);

/* d = (L L^T)^-1 gamma, E = 1/2 gamma.d (E is a device scalar), by blocked substitution (panels
 * of 64: the diagonal block in shared memory, the rest of the right-hand side updated by row-parallel
 * panel products). Replaces df_coulomb_solve with cholV (gs_dft/coulomb/ri.py:472-482). */
size_t gsdft_j_solve_workspace_size(int64_t n_aux);
int gsdft_j_solve(const double* L, const double* gamma, int64_t n_aux, double* d, double* E,
                  void* ws, size_t ws_bytes, gsdft_stream_t stream);

/* The same solve through the inverse factor, for repeated steps on one factor.
 * gsdft_j_solve_inverse (once per refresh) writes Linv (n_aux, n_aux), row-major and packed: its
 * lower triangle with the diagonal is L^-1 and its strict upper triangle is that of L^-T (the
 * mirror of the strict lower one), from the lower factor L (n_aux <= GSDFT_SOLVE_INV_MAX; one n_aux^2
 * buffer, 22.5 GB at n_aux = 53,000; computed on the tensor cores by recursive doubling).
 * gsdft_j_solve_inv then gives d = L^-T (L^-1 gamma) as two row-parallel triangular mat-vecs that
 * read the packed matrix once, with no sequential substitution and no library call. With the factor
 * L (non-NULL) it adds one step of iterative refinement, r = gamma - L (L^T d), d += L^-T L^-1 r,
 * and E = 1/2 gamma.d: the result then matches a substitution solve (gsdft_j_solve) to the
 * accuracy of a backward-stable solve, where the multiplication by a computed inverse alone carries
 * errors of order cond(L) times the unit roundoff; this streams the factor and the inverse twice
 * each. With L = NULL, E = 1/2 |L^-1 gamma|^2. Replaces, per step, cho_solve in df_coulomb_solve
 * (gs_dft/coulomb/ri.py:472-482). */
#define GSDFT_SOLVE_INV_MAX 65536
int gsdft_j_solve_inverse(const double* L, int64_t n_aux, double* Linv, gsdft_stream_t stream);
size_t gsdft_j_solve_inv_workspace_size(int64_t n_aux);
int gsdft_j_solve_inv(const double* Linv, const double* L, const double* gamma, int64_t n_aux,
                      double* d, double* E, void* ws, size_t ws_bytes, gsdft_stream_t stream);

/* Reverse pass over (representative x aux): with dbar = g_E * d (g_E device scalar, NULL = 1), the
 * per-pair sums, (n_rep, GSDFT_VJP_FIELDS), from which J_a = sum_P (P|a) dbar_P and the cotangents
 * of A_hat, P, KN follow. Replaces the node reverse nodes_bwd and the eigh / dp2 autodiff
 * (gs_dft/coulomb/ri.py:145-147,190-222). */
size_t gsdft_j_vjp_workspace_size(int64_t n_rep, int64_t n_aux);
int gsdft_j_vjp(const double* rec, int64_t n_rep, const double* beta, const double* R,
                const double* KN, const double* d, const double* g_E, int64_t n_aux,
                double* sums, void* ws, size_t ws_bytes, gsdft_stream_t stream);

/* Chain per representative: sums -> cotangents of A_hat, P, KN -> per-side (A_i, mu_i, N_i), (A_j, mu_j,
 * N_j) contributions side (n_rep, GSDFT_SIDE_FIELDS); J (n, list order: written at each
 * representative's position and at its merged transpose's; 0 on zero-weight entries); jw (n_rep)
 * = J times the representative's summed weight, the factor of q's gradient. The reverse of
 * gs_dft/coulomb/stream.py:203-215. sums (gsdft_j_vjp's layout) and xc (GSDFT_XC_FIELDS per
 * representative, cotangents given directly, e.g. by gsdft_exact_j_vjp) are each optional (NULL)
 * and add. */
int gsdft_pair_chain(const double* A9, const double* mu, const double* N, int64_t M,
                     const int32_t* pi, const int32_t* pj, const int32_t* rep_pos,
                     const int32_t* rep_twin, const double* rep_w, int64_t n_rep, int64_t n,
                     const double* rec, const double* sums, const double* xc, double* side,
                     double* J, double* jw, gsdft_stream_t stream);

/* Deterministic per-splat sums of the side contributions (plan groupings) -> gA6 (M,6), gmu (M,3),
 * gN (M). Replaces the segment scatter of JAX autodiff through A[pi], A[pj]. */
int gsdft_splat_reduce(const double* side, const int32_t* order_i, const int64_t* seg_i,
                       const int32_t* order_j, const int64_t* seg_j, int64_t n_rep, int64_t M,
                       double* gA6, double* gmu, double* gN, gsdft_stream_t stream);

/* g_C[i,o] = occ_o (sum_{a: pi=i} J_a w_a C[pj_a,o] + sum_{a: pj=i} J_a w_a C[pi_a,o]): the gradient
 * through q_a (gs_dft/coulomb/ri.py:456). jw from gsdft_pair_chain; groupings and partners from
 * gsdft_pair_groups. Summed in a fixed order (bitwise reproducible). */
int gsdft_density_grad(const int32_t* order_i, const int64_t* seg_i, const int32_t* partner_i,
                       const int32_t* order_j, const int64_t* seg_j, const int32_t* partner_j,
                       const double* jw, int64_t n_rep, int64_t M, const double* C_occ,
                       const double* occ, int64_t n_occ, double* g_C, gsdft_stream_t stream);

/* The same q and g_C for many orbitals, as dense tiles on the FP64 tensor cores. The splats are cut
 * into n_blocks = ceil(M / 64) row blocks; block b has the sorted partner list
 * jidx[joff[b] .. joff[b] + nj[b]) (the splats paired with its rows) and a dense tile of
 * rows_b x nj[b] doubles at buf + boff[b] (rows_b = min(64, M - 64 b)); representative a's cell is
 * cell[a] (its row splat's row, its partner's column).
 * gsdft_block_density: tile_b = (C_I diag(occ)) C_J^T (an SDDMM over the block, max_nj = max nj[b]),
 * then q_a = rep_w[a] tile[cell[a]] into rec (Q and QK) for the n_rep representatives.
 * gsdft_block_density_grad: zeroes buf (buf_len doubles), scatters vals[a] (J w) to cell[a], and sets
 * g_C = beta g_C + tile (C_J diag(occ)) row block by row block (an SpMM). Called for the by-pi
 * grouping (beta = 0) then the by-pj grouping (beta = 1), it gives gsdft_density_grad's g_C.
 * Deterministic. Replaces the same expressions as gsdft_pair_prep's q (gs_dft/coulomb/ri.py:456) and
 * gsdft_density_grad (its gradient); the grouping is refresh-time state of the host layer. */
int gsdft_block_density(const double* C_occ, const double* occ, int64_t M, int64_t n_occ,
                        int64_t n_blocks, const int64_t* boff, const int32_t* nj, const int64_t* joff,
                        const int32_t* jidx, int64_t max_nj, const int64_t* cell,
                        const double* rep_w, int64_t n_rep, double* buf, double* rec,
                        gsdft_stream_t stream);
int gsdft_block_density_grad(const double* vals, const int64_t* cell, int64_t n_rep,
                             const double* C_occ, const double* occ, int64_t M, int64_t n_occ,
                             int64_t n_blocks, const int64_t* boff, const int32_t* nj,
                             const int64_t* joff, const int32_t* jidx, int64_t buf_len,
                             double* buf, double beta, double* g_C, gsdft_stream_t stream);

/* Screened nuclear attraction on the pair representatives: V_a = -2 pi KN_a sum_A Z_A sum_t w_t
 * det(A_hat + t^2 I)^-1/2 exp(-t^2 d.A_hat (A_hat + t^2 I)^-1 d), d = R_A - P_a, and
 * E_ne = sum_a q_a V_a (q from rec, so pair weights and twin merging apply). Replaces
 * _full_nuclear_pairs / screened_nuclear_pairs / screened_external_energy
 * (gs_dft/screening/pairs.py:348-370, 378-380, 409-440). atoms (n_atoms, 4) row-major = (x, y, z, Z),
 * 32-byte aligned; E a device scalar (always written). V (optional): each representative's V at
 * rep_pos[a] and, when rep_twin[a] >= 0, at rep_twin[a] of a list of length n (zero elsewhere), or at
 * a when rep_pos is NULL. sums (optional): the reverse-pass sums of g_E * E_ne (g_E a device scalar,
 * NULL = 1) in gsdft_j_vjp's layout and scale, written (add = 0) or added (add = 1: onto gsdft_j_vjp's,
 * so one gsdft_pair_chain carries E_J + E_ne and its J is dE/dq including V). Deterministic. */
size_t gsdft_vne_workspace_size(int64_t n_rep);
int gsdft_vne(const double* rec, int64_t n_rep, const double* atoms, int64_t n_atoms,
              const double* g_E, const int32_t* rep_pos, const int32_t* rep_twin, int64_t n,
              double* V, double* E, double* sums, int add, void* ws, size_t ws_bytes,
              gsdft_stream_t stream);

/* P_a = sum_o occ_o C_occ[pi_a, o] C_occ[pj_a, o] for every listed pair (no weights), the density
 * matrix entries on the pair list without forming P. Replaces density_pairs
 * (gs_dft/screening/pairs.py:403-406). */
int gsdft_density_pairs(const int32_t* pi, const int32_t* pj, int64_t n, const double* C_occ,
                        const double* occ, int64_t n_occ, double* P, gsdft_stream_t stream);

/* The reverse pass of E = sum_{P,a} W[P][a] (P|a): gsdft_j_vjp with a per-(aux, pair) weight matrix
 * Wt, stored aux-major (n_aux rows of leading dimension ldw >= n_rep: Wt[P * ldw + a]), instead of
 * dbar_P q_a; the sums then go to gsdft_pair_chain with records whose q is 1 (gsdft_k_unit_q). Used
 * by the RI-K gradient (the reference differentiates gs_dft/coulomb/ri.py:497-544 with JAX
 * autodiff). */
size_t gsdft_j_vjp_weighted_workspace_size(int64_t n_rep, int64_t n_aux);
int gsdft_j_vjp_weighted(const double* rec, int64_t n_rep, const double* beta, const double* R,
                         const double* KN, const double* Wt, int64_t ldw, int64_t n_aux,
                         const double* nodes, int n_nodes, double* sums, void* ws, size_t ws_bytes,
                         gsdft_stream_t stream);

/* A runtime node rule of the 3-centre kernels (for the weighted reverse pass and RI-K): Gauss-Legendre
 * on [0, upper] with n_nodes <= 20 nodes (ascending), the rule of the long-range kernel
 * erf(omega r)/r with upper = omega (_gauss_legendre_segment / _lr_nodes,
 * gs_dft/integrals/dense.py:56-76, gs_dft/coulomb/ri.py:232-235; the reference uses 12 nodes).
 * table (GSDFT_NODE_TABLE_DOUBLES doubles, device): t^2 of each node (20 slots), t^4 (20 slots),
 * then per node 64 entries w_n 2^(j/64). Nodes by Newton's method on P_n in FP64. Node screening
 * does not apply to a runtime rule (its weights are not monotone). */
#define GSDFT_NODE_TABLE_DOUBLES 1320
int gsdft_lr_node_table(double upper, int n_nodes, double* table, gsdft_stream_t stream);

/* The long-range aux metric (P|erf(omega r)/r|Q): F0(T) -> sqrt(z) F0(z T), z = omega^2 /
 * (omega^2 + rho) (coulomb_block with omega, gs_dft/coulomb/ri.py:63-101,267-275). omega > 0. */
int gsdft_aux_metric_lr(const double* beta, const double* R, const double* KN, int64_t n_aux,
                        double omega, double* V, gsdft_stream_t stream);

/* Screened RI-K over the pair representatives: D[P,o,o'] = sum_{live (i,k)} (P|ik) C_io C_ko',
 * E_K = -tr((V + lam I)^-1 D D^T) = -|L^-1 D|^2 (replaces _exchange_M_streamed_screened and
 * df_exchange_energy_screened, gs_dft/coulomb/ri.py:497-544). The pair list must be an ordered 0/1
 * list (the reference masks with valid & occupied); a merged transposed twin adds C_ko C_io'. Linv is
 * the packed inverse factor of gsdft_j_solve_inverse (its lower triangle L^-1 is read). nodes NULL:
 * the 1/r kernel; a gsdft_lr_node_table rule (with the factor of gsdft_aux_metric_lr's metric): the
 * long-range exchange E_K[erf(omega r)/r]. The orbital products are streamed in chunks of occ_chunk
 * orbitals (0 = all at once; the reference's occ_chunk): the workspace (gsdft_k_workspace_size)
 * holds the integral block (8 n_rep n_aux bytes), one chunk of products (8 n_rep occ_chunk n_occ
 * bytes), n_aux x n_occ^2 doubles and a chunk of D with its split partials. Writes Z = L^-1 D
 * (n_aux x n_occ^2, row-major; kept for the backward) and E (device scalar). The contractions are
 * the library's DMMA GEMMs. Pass the same, untouched workspace to gsdft_k_backward. */
size_t gsdft_k_workspace_size(int64_t n_rep, int64_t n_aux, int64_t n_occ, int64_t occ_chunk);
int gsdft_k_forward(const double* rec, const int32_t* pi, const int32_t* pj, const int32_t* rep_pos,
                    const int32_t* rep_twin, int64_t n_rep, const double* beta, const double* R,
                    const double* KN, int64_t n_aux, const double* nodes, int n_nodes,
                    const double* Linv, const double* C_occ, int64_t n_occ, int64_t occ_chunk,
                    double* Z, double* E, void* ws, size_t ws_bytes, gsdft_stream_t stream);
/* Gradient of g_E * E_K (g_E a device scalar, NULL = 1): the reverse-pass sums (for gsdft_pair_chain
 * with gsdft_k_unit_q records) and g_C (M x n_occ, written). Groupings and partners from
 * gsdft_pair_groups. Overwrites the workspace's integral block: a second backward needs the forward
 * again. Deterministic. */
int gsdft_k_backward(const double* rec, const int32_t* pi, const int32_t* pj,
                     const int32_t* rep_pos, const int32_t* rep_twin, int64_t n_rep,
                     const double* beta, const double* R, const double* KN, int64_t n_aux,
                     const double* nodes, int n_nodes, const double* Linv, const double* C_occ,
                     int64_t n_occ, int64_t occ_chunk, const double* Z,
                     const double* g_E, const int32_t* order_i, const int64_t* seg_i,
                     const int32_t* partner_i, const int32_t* order_j, const int64_t* seg_j,
                     const int32_t* partner_j, int64_t M, double* sums, double* g_C, void* ws,
                     size_t ws_bytes, gsdft_stream_t stream);
/* rec_out = rec with q = 1 (Q = 1, QK = KN pref), for the chain of a weighted reverse pass. */
int gsdft_k_unit_q(const double* rec, int64_t n_rep, double* rec_out, gsdft_stream_t stream);

/* Quadrature rules of the exact (pair|pair) integral: the 20-node half-line rule of the Schur block
 * (full_eri_block_schur, gs_dft/coulomb/stream.py:249-283) and the 32-node Boys-scaled rule of the
 * fused block (full_eri_block_fused, :323-458: nodes t^2 = rho c_k with a per-(a, b) scale rho). */
enum { GSDFT_EXACT_SCHUR20 = 0, GSDFT_EXACT_FUSED32 = 1 };

/* Screened exact Hartree energy E_J = 1/2 sum_{a,b} q_a q_b (a|b) over the pair representatives
 * (q from rec: pair weights, densities and merged twins included), (a|b) the exact 6-D Coulomb
 * integral of two product Gaussians on the given rule. Replaces screened_coulomb_energy
 * (gs_dft/coulomb/stream.py:294-320) with either block. Writes J (n_rep: J_a = sum_b q_b (a|b)) and
 * E (device scalar). O(n_rep^2). Deterministic. The workspace size covers both rules. */
size_t gsdft_exact_j_workspace_size(int64_t n_rep);
int gsdft_exact_j(const double* rec, int64_t n_rep, int rule, double* J, double* E, void* ws,
                  size_t ws_bytes, gsdft_stream_t stream);

/* Reverse pass of g_E * E_J (g_E a device scalar, NULL = 1) of gsdft_exact_j: per representative the
 * cotangents of A_hat, P and KN and dE/dq into xc (n_rep, GSDFT_XC_FIELDS), for gsdft_pair_chain
 * (sums NULL, or V_ne's). Each (a, b) evaluates dF/dH and dF/dd of the node sum in closed form over
 * the same nodes (and, for the fused rule, the derivative through its per-(a, b) scale): the
 * derivative the reference takes by autodiff of the streamed blocks with the fused rule's
 * hand-written node VJP (gs_dft/coulomb/stream.py:144-189, 294-320, 356-398). O(n_rep^2).
 * Deterministic. */
size_t gsdft_exact_j_vjp_workspace_size(int64_t n_rep);
int gsdft_exact_j_vjp(const double* rec, int64_t n_rep, int rule, const double* g_E, double* xc,
                      void* ws, size_t ws_bytes, gsdft_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* GSDFT_B200_H */
