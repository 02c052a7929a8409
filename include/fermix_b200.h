/* fermix_b200: batched slogdet / slogpf / det / pf on NVIDIA B200 (sm_100a).
 *
 * C ABI of libfermix_b200.so. Plain pointers and sizes only. Every entry point is
 * stream-ordered (no host synchronisation), allocates nothing, and returns 0 or one of
 * the FX_ERR_* codes; numerical singularity is not an error (it gives sign 0 and
 * logabs -inf). The caller owns all memory: inputs, outputs and the optional
 * workspace (size from fermix_workspace_bytes: the blocked engines for n > 256 keep
 * their matrices there, a slice of the batch at a time; smaller n uses it only when a
 * matrix does not fit in one block's shared memory).
 *
 * Arrays are C-contiguous: a (batch, n, n) row-major, complex values interleaved
 * (re, im) as in numpy / torch / XLA; sign, value and coef have the input dtype,
 * logabs the real dtype.
 *
 * Reference interfaces these entry points replace (ChenAo-Phys/fermix, paths relative
 * to that project; the reference reaches its kernels through pl.pallas_call, wrapped by
 * _pcall in src/fermix/_field.py:357-389):
 *   fermix_slogdet       <- _slogdet_core / _lu_core       src/fermix/_diff.py:42-49, src/fermix/_lu.py:543-611
 *   fermix_slogdet_grad  <- _parts / _lu_parts, _det_gradT src/fermix/_diff.py:62-77, src/fermix/_inverse.py:502-531,
 *                                                          src/fermix/_diff.py:205-246
 *   fermix_slogpf        <- _slogpf_core / _pf_core        src/fermix/_diff.py:52-59, src/fermix/_pf.py:497-502
 *   fermix_slogpf_grad   <- _pf_grad_parts / _pf_parts     src/fermix/_diff.py:80-89, src/fermix/_pfinv.py:196-269
 *   fermix_workspace_bytes, fermix_strerror, fermix_check_prec
 *                        <- Field.check_prec / PREC        src/fermix/_field.py:20-23, :262-275
 */
#ifndef FERMIX_B200_H
#define FERMIX_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* dtype codes (src/fermix/_field.py:24-29, KINDS) */
#define FX_F32 0
#define FX_F64 1
#define FX_C64 2
#define FX_C128 3

/* prec codes (src/fermix/_field.py:20-23, PREC): 0 = the dtype's default
 * ("tf32x3" for float32 / complex64, "ieee" otherwise) */
#define FX_PREC_DEFAULT 0
#define FX_PREC_TF32X3 1
#define FX_PREC_IEEE 2

/* ops for fermix_workspace_bytes */
#define FX_OP_SLOGDET 0
#define FX_OP_SLOGPF 1

/* error codes */
#define FX_OK 0
#define FX_ERR_DTYPE 1     /* unsupported dtype code */
#define FX_ERR_SHAPE 2     /* batch < 0 or n < 0 (or n too large for int indexing) */
#define FX_ERR_PREC 3      /* prec unknown, or tf32x3 with a 64-bit dtype */
#define FX_ERR_WORKSPACE 4 /* workspace missing or smaller than one matrix slot */
#define FX_ERR_NULL 5      /* a required pointer is NULL */
#define FX_ERR_CUDA 6      /* a CUDA launch / attribute call failed */
#define FX_ERR_DEVICE 7    /* no usable CUDA device */
#define FX_ERR_TIMEOUT 8   /* a bounded wait inside a kernel gave up (reported by fermix_device_status) */

/* (sign, logabs) of each matrix; value = sign * exp(logabs) (det) or, for n <= 4, the
 * explicit polynomial. value may be NULL. Replaces _slogdet_core / _lu_core. */
int fermix_slogdet(void* stream, int dtype, int prec, int64_t batch, int64_t n, const void* a, void* sign,
                   void* logabs, void* value, void* workspace, size_t workspace_bytes);

/* The forward plus the gradient matrix of each member, scaled by coef[b] (NULL = 1) and
 * conjugated when conj_out != 0:
 *   adjugate == 0: grad = coef * A^-T (slogdet; zero for an exactly singular or
 *                  non-finite member)            -- _lu_parts, src/fermix/_inverse.py:502-531
 *   adjugate != 0: grad = coef * adj(A)^T (det; finite for singular A, exact for up to two
 *                  zero pivots)                  -- _det_gradT, src/fermix/_diff.py:205-246
 * (sign, logabs, value) are bit-identical to fermix_slogdet on the same input. */
int fermix_slogdet_grad(void* stream, int dtype, int prec, int64_t batch, int64_t n, const void* a,
                        const void* coef, int conj_out, int adjugate, void* sign, void* logabs, void* value,
                        void* grad, void* workspace, size_t workspace_bytes);

/* (sign, logabs) of the Pfaffian of S = (a - a^T) / 2 (skew_symmetrize != 0) or of the
 * skew input a itself; odd n gives (0, -inf). Replaces _slogpf_core / _pf_core. */
int fermix_slogpf(void* stream, int dtype, int prec, int64_t batch, int64_t n, int skew_symmetrize, const void* a,
                  void* sign, void* logabs, void* value, void* workspace, size_t workspace_bytes);

/* The forward plus the gradient w.r.t. a of each member, scaled by coef[b]:
 *   adjugate == 0: grad = coef * S^-T / 2 = -coef * S^-1 / 2 (slogpf; zero for an exactly
 *                  singular member)              -- _pf_parts(adjugate=False)
 *   adjugate != 0: grad = coef * pf(S) S^-T / 2 (pf; the Pfaffian adjugate, finite for
 *                  singular S)                   -- _pf_parts(adjugate=True), src/fermix/_pfinv.py:196-269
 * Odd n gives a zero gradient. (sign, logabs, value) equal fermix_slogpf bit for bit. */
int fermix_slogpf_grad(void* stream, int dtype, int prec, int64_t batch, int64_t n, int skew_symmetrize,
                       const void* a, const void* coef, int conj_out, int adjugate, void* sign, void* logabs,
                       void* value, void* grad, void* workspace, size_t workspace_bytes);

/* Complex input and gradient as split real / imaginary planes (no separate reference entry:
 * the reference computes complex values as real planes, Field.split / join,
 * src/fermix/_field.py:246-256, and its kernels take the planes as separate operands,
 * _pcall src/fermix/_field.py:357-389). dtype is FX_C64 or FX_C128 (else FX_ERR_DTYPE);
 * a_re / a_im (and grad_re / grad_im) are (batch, n, n) arrays of the real type; sign and
 * value stay interleaved complex (batch,) arrays, logabs real. Otherwise as the
 * interleaved entry points, with the same results bit for bit. For n > 256 (slogdet, and
 * slogpf with even n <= 8192) forward and slog gradient read and write the planes
 * directly; other cases pass through the workspace in chunks of about 1 GiB. Workspace:
 * fermix_workspace_bytes_planar. */
int fermix_slogdet_planar(void* stream, int dtype, int prec, int64_t batch, int64_t n, const void* a_re,
                          const void* a_im, void* sign, void* logabs, void* value, void* workspace,
                          size_t workspace_bytes);
int fermix_slogdet_grad_planar(void* stream, int dtype, int prec, int64_t batch, int64_t n, const void* a_re,
                               const void* a_im, const void* coef, int conj_out, int adjugate, void* sign,
                               void* logabs, void* value, void* grad_re, void* grad_im, void* workspace,
                               size_t workspace_bytes);
int fermix_slogpf_planar(void* stream, int dtype, int prec, int64_t batch, int64_t n, int skew_symmetrize,
                         const void* a_re, const void* a_im, void* sign, void* logabs, void* value, void* workspace,
                         size_t workspace_bytes);
int fermix_slogpf_grad_planar(void* stream, int dtype, int prec, int64_t batch, int64_t n, int skew_symmetrize,
                              const void* a_re, const void* a_im, const void* coef, int conj_out, int adjugate,
                              void* sign, void* logabs, void* value, void* grad_re, void* grad_im, void* workspace,
                              size_t workspace_bytes);
size_t fermix_workspace_bytes_planar(int op, int dtype, int64_t batch, int64_t n, int grad);

/* slogdet of gathered matrices (no reference counterpart; the fused gather of the QMC
 * caller in the reference's README): matrix b is rows occ[b * n + i] (int32, i < n) of phi
 * (phi_rows x phi_ld row-major, same dtype), columns 0 .. n - 1, so that the batch is
 * never materialised. grad == NULL: the forward of fermix_slogdet; otherwise also the
 * per-matrix gradient coef * A^-T as fermix_slogdet_grad (adjugate 0). An index outside
 * [0, phi_rows) makes that matrix NaN. Results equal fermix_slogdet / _grad on the
 * materialised batch bit for bit. Workspace: fermix_slogdet_gather_workspace_bytes (0 for
 * float32 tf32x3 with 8 <= n <= 256, where the tensor-memory kernel reads the rows). */
int fermix_slogdet_gather(void* stream, int dtype, int prec, int64_t batch, int64_t n, const void* phi,
                          int64_t phi_rows, int64_t phi_ld, const int* occ, const void* coef, int conj_out,
                          void* sign, void* logabs, void* value, void* grad, void* workspace,
                          size_t workspace_bytes);
size_t fermix_slogdet_gather_workspace_bytes(int dtype, int prec, int64_t batch, int64_t n, int grad);

/* Rank-k row replacement from the exported inverse (no reference counterpart; the
 * single- and multi-electron moves of a QMC caller, built on the inverse that
 * fermix_slogdet_grad exports -- _lu_parts, src/fermix/_inverse.py:502-531). g holds
 * G = A^-T per matrix (fermix_slogdet_grad with coef NULL, conj_out 0, adjugate 0). A move
 * replaces rows idx[b * k + r] (int32, distinct, in [0, n)) of A by rows[b, r, :]
 * ((batch, k, n), same dtype), 0 <= k <= 16, k <= n.
 *   fermix_slogdet_ratio:  (sign, logabs) of det(A') / det(A) = det(U A^-1 E), in the
 *                          slogdet conventions (sign in the input dtype; a singular ratio
 *                          gives (0, -inf); an index outside [0, n) gives NaN). Reads k
 *                          rows of each G; no workspace.
 *   fermix_slogdet_update: the same ratio, and G replaced in place by A'^-T (Woodbury) for
 *                          every matrix with accept[b] != 0 (accept NULL = all). A member
 *                          whose ratio is exactly 0 gets G' = 0, one with a bad index keeps
 *                          G. rows must not overlap g. Workspace:
 *                          fermix_slogdet_update_workspace_bytes. */
int fermix_slogdet_ratio(void* stream, int dtype, int64_t batch, int64_t n, int64_t k, const void* g,
                         const void* rows, const int* idx, void* sign, void* logabs);
int fermix_slogdet_update(void* stream, int dtype, int64_t batch, int64_t n, int64_t k, void* g, const void* rows,
                          const int* idx, const unsigned char* accept, void* sign, void* logabs, void* workspace,
                          size_t workspace_bytes);
size_t fermix_slogdet_update_workspace_bytes(int dtype, int64_t batch, int64_t n, int64_t k);

/* One-index Pfaffian move (no reference counterpart; the one-electron move of a Pfaffian
 * wavefunction, on the gradient fermix_slogpf_grad exports -- _pf_parts,
 * src/fermix/_pfinv.py:196-269). g holds G = S^-T / 2 per matrix (fermix_slogpf_grad with
 * coef NULL, conj_out 0, adjugate 0). The move replaces row idx[b] of the skew S by
 * row[b, :] ((batch, n), same dtype) and column idx[b] by -row[b, :]; row[b, idx[b]] is
 * ignored (the diagonal stays 0). n >= 2.
 *   fermix_slogpf_ratio:  (sign, logabs) of pf(S') / pf(S) = 2 G_i . u in the slogpf
 *                         conventions (0, -inf when it is 0; NaN for an index outside
 *                         [0, n)). Reads one row of each G; no workspace.
 *   fermix_slogpf_update: the same ratio, and G replaced in place by S'^-T / 2 (rank-2 skew
 *                         Woodbury) for every matrix with accept[b] != 0 (accept NULL = all);
 *                         a member whose ratio is exactly 0 gets G' = 0, one with a bad index
 *                         keeps G. row must not overlap g. Workspace:
 *                         fermix_slogpf_update_workspace_bytes. */
int fermix_slogpf_ratio(void* stream, int dtype, int64_t batch, int64_t n, const void* g, const void* row,
                        const int* idx, void* sign, void* logabs);
int fermix_slogpf_update(void* stream, int dtype, int64_t batch, int64_t n, void* g, const void* row, const int* idx,
                         const unsigned char* accept, void* sign, void* logabs, void* workspace,
                         size_t workspace_bytes);
size_t fermix_slogpf_update_workspace_bytes(int dtype, int64_t batch, int64_t n);

/* k-index Pfaffian move (no reference counterpart; the multi-electron move of a Pfaffian
 * wavefunction, on the gradient fermix_slogpf_grad exports -- _pf_parts,
 * src/fermix/_pfinv.py:196-269). g holds G = S^-T / 2 per matrix. The move replaces rows
 * idx[b * k + r] (int32, distinct, in [0, n)) of the skew S by rows[b, r, :] ((batch, k, n))
 * and the same columns by -rows[b, r, :], applied in order r = 0 .. k - 1: it is the
 * composition of k one-index moves (on the idx x idx block the later row wins; rows[b, r,
 * idx[b * k + r]] is ignored). 0 <= k <= 16, k <= n, n >= 2.
 *   fermix_slogpf_ratio_k:  (sign, logabs) of pf(S') / pf(S), in the slogpf conventions
 *                           ((0, -inf) when it is 0, NaN for an index outside [0, n)).
 *                           Reads all of G once (the ratio depends on u_r^T G u_s).
 *   fermix_slogpf_update_k: the same ratio, and G replaced in place by S'^-T / 2 for every
 *                           matrix with accept[b] != 0 (accept NULL = all); a member whose
 *                           ratio is exactly 0 gets G' = 0, one with a bad index keeps G.
 *                           rows must not overlap g. G is read twice and written once.
 * Both take a workspace of fermix_slogpf_move_k_workspace_bytes. */
int fermix_slogpf_ratio_k(void* stream, int dtype, int64_t batch, int64_t n, int64_t k, const void* g,
                          const void* rows, const int* idx, void* sign, void* logabs, void* workspace,
                          size_t workspace_bytes);
int fermix_slogpf_update_k(void* stream, int dtype, int64_t batch, int64_t n, int64_t k, void* g, const void* rows,
                           const int* idx, const unsigned char* accept, void* sign, void* logabs, void* workspace,
                           size_t workspace_bytes);
size_t fermix_slogpf_move_k_workspace_bytes(int dtype, int64_t batch, int64_t n, int64_t k);

/* Size of the fixed device array fermix_slogdet_grad_static uses instead of a workspace
 * (16 MiB, one copy per device, part of the library's device image). */
#define FX_STATIC_SCRATCH_BYTES (16u << 20)

/* fermix_slogdet_grad without a workspace argument (no reference counterpart): the LU
 * kernels take their per-block matrix slots from a fixed device array of
 * FX_STATIC_SCRATCH_BYTES instead of caller memory, and the call allocates nothing. For
 * callers that cannot allocate device memory when they call: a host framework whose
 * allocator owns the device and passes the op no scratch operand, or a latency-bound loop
 * where cudaMalloc / cudaFree would synchronise the device.
 * Limit: one slot (2 n^2 elements, needed when a matrix does not fit in one block's shared
 * memory) must fit in the array -- n <= 1448 (float32), 1024 (float64, complex64), 724
 * (complex128); larger n returns FX_ERR_WORKSPACE. Fewer slots than resident blocks means
 * fewer blocks in flight, so large-n calls run slower than fermix_slogdet_grad with a full
 * workspace. Results are bit-identical to fermix_slogdet_grad.
 * The array is shared by all calls on a device: calls that overlap in time on one device
 * (different streams or host threads) race on it; serialise them. The first call on each
 * device looks the array up (cudaGetSymbolAddress) and should come before any stream
 * capture. */
int fermix_slogdet_grad_static(void* stream, int dtype, int prec, int64_t batch, int64_t n, const void* a,
                               const void* coef, int conj_out, int adjugate, void* sign, void* logabs, void* value,
                               void* grad);

/* Status of the library's kernels on the current device (no reference counterpart):
 * FX_OK, or FX_ERR_TIMEOUT when a kernel gave up one of its bounded waits (a tensor-core
 * completion or a bulk copy that did not arrive) since the status was last cleared. The
 * members such a kernel was working on got NaN outputs; the kernel waited once more, with
 * the default limit, for the operation in flight before it released tensor memory and
 * returned, so the context stays usable. Entry points are stream-ordered and cannot
 * return this code themselves. This call synchronises the device first; clear != 0 resets
 * the status to FX_OK. Returns FX_ERR_CUDA / FX_ERR_DEVICE if the status cannot be read. */
int fermix_device_status(int clear);

/* Polls of each bounded wait in the library's kernels, for launches issued after the call
 * (process-wide; no reference counterpart). FX_WAIT_POLLS_DEFAULT is the default; 0 makes
 * every such wait give up at once, which tests of the timeout path use. Returns the
 * previous value. */
#define FX_WAIT_POLLS_DEFAULT (1u << 26)
unsigned fermix_set_wait_polls(unsigned polls);

/* Workspace bytes a call needs on the current device (0 when every matrix fits in one
 * block's shared memory); grad != 0 for the *_grad entry points. */
size_t fermix_workspace_bytes(int op, int dtype, int64_t batch, int64_t n, int grad);

/* FX_OK when prec is valid for dtype (Field.check_prec, src/fermix/_field.py:265-275). */
int fermix_check_prec(int dtype, int prec);

/* Static description of an error code. */
const char* fermix_strerror(int code);

/* Self-test of the tensor-core path on the current GPU (no reference counterpart): one
 * 128 x 128 x 16 update d = (accumulate ? c : 0) + (negate ? -1 : 1) * a b^T computed with
 * tcgen05 3xTF32 MMAs into tensor memory, all operands row-major float32 (a, b: 128 x 16;
 * c, d: 128 x 128; device pointers). disable_lanes (host array of 4 words, or NULL): bit l
 * of word w keeps row 32 w + l of d equal to c. *status (device) gets bit 0 set if the
 * MMA completion wait timed out. */
int fermix_selftest_umma(void* stream, const float* a, const float* b, const float* c, float* d, int negate,
                         int accumulate, const unsigned* disable_lanes, int* status);

/* FMA-pipe throughput probe (no reference counterpart; it measures the FP32 / FP64 FMA
 * peaks the benchmark's compute roofline divides by): blocks x 256 threads, each running 8
 * independent FMA chains of iters steps, 16 * iters flops per thread. dtype FX_F32 or
 * FX_F64; out is a device scratch word of that type (written only in a case that does not
 * occur). Time it with events on the stream. */
int fermix_selftest_fma_rate(void* stream, int dtype, int blocks, int iters, void* out);

/* Library version, major * 10000 + minor * 100 + patch. */
int fermix_version(void);

#ifdef __cplusplus
}
#endif

#endif /* FERMIX_B200_H */
