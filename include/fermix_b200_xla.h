/* fermix_b200 XLA custom-call adapter (part of libfermix_b200.so).
 *
 * The reference enters its kernels from jitted JAX functions: _slogdet / _slogpf
 * (src/fermix/api.py:110-145) reach the Pallas drivers through the custom_jvp rules of
 * src/fermix/_diff.py (the kernel branch is picked by lax.platform_dependent,
 * src/fermix/_diff.py:35-39). To put this library under those functions, JAX registers one
 * target with the legacy custom-call ABI, which needs no XLA headers:
 *
 *     jax.ffi.register_ffi_target("fermix_b200", jax.ffi.pycapsule(lib.fermix_xla_custom_call),
 *                                 platform="CUDA", api_version=0)
 *
 * and calls it through jax.ffi.ffi_call(..., legacy_backend_config=<descriptor bytes>).
 * XLA owns every buffer, passes them as one array of device pointers in the order below,
 * and launches on its own stream; the scratch the library needs is one more (uint8)
 * output buffer of descriptor.workspace_bytes.
 *
 * Buffer order (inputs first, then outputs, as XLA lists them):
 *   FX_XLA_SLOGDET / FX_XLA_SLOGPF:           a, sign, logabs, [value], [workspace]
 *   FX_XLA_SLOGDET_GRAD / FX_XLA_SLOGPF_GRAD: a, [coef], sign, logabs, [value], grad, [workspace]
 * where [value] is present when flags & FX_XLA_VALUE, [coef] when flags & FX_XLA_COEF and
 * [workspace] when workspace_bytes > 0. The arguments mean what they mean for the C entry
 * point of the same name (include/fermix_b200.h).
 */
#ifndef FERMIX_B200_XLA_H
#define FERMIX_B200_XLA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FX_XLA_MAGIC 0x46584231u /* "FXB1" */
#define FX_XLA_VERSION 1

/* descriptor ops */
#define FX_XLA_SLOGDET 0
#define FX_XLA_SLOGDET_GRAD 1
#define FX_XLA_SLOGPF 2
#define FX_XLA_SLOGPF_GRAD 3

/* descriptor flags */
#define FX_XLA_VALUE 1u    /* a value output follows logabs */
#define FX_XLA_COEF 2u     /* a coef input follows a (gradient ops) */
#define FX_XLA_CONJ_OUT 4u /* gradient ops: conj_out */
#define FX_XLA_ADJUGATE 8u /* gradient ops: adjugate */
#define FX_XLA_SKEW 16u    /* slogpf ops: skew_symmetrize */

/* The opaque bytes of one custom call (little-endian, 48 bytes, no padding). */
typedef struct {
  uint32_t magic;   /* FX_XLA_MAGIC */
  int32_t version;  /* FX_XLA_VERSION */
  int32_t op;       /* FX_XLA_* op */
  int32_t dtype;    /* FX_F32 .. FX_C128 */
  int32_t prec;     /* FX_PREC_* */
  uint32_t flags;   /* FX_XLA_* flags */
  int64_t batch;
  int64_t n;
  uint64_t workspace_bytes; /* size of the workspace buffer (0: none) */
} fermix_xla_descriptor;

/* Legacy (api_version 0) custom-call target: unpacks the descriptor and the buffer array and
 * calls the matching entry point on XLA's stream. That ABI has no status channel, so a
 * non-zero status (a malformed descriptor or any FX_ERR_* of the entry point) is recorded
 * for fermix_xla_last_error and the outputs are left unwritten. Replaces the pallas_call
 * dispatch of _pcall (src/fermix/_field.py:357-389) for the four core ops. */
void fermix_xla_custom_call(void* stream, void** buffers, const char* opaque, size_t opaque_len);

/* The first non-zero status a custom call recorded since the last clear (0 if none);
 * clear != 0 resets it. Process-wide. */
int fermix_xla_last_error(int clear);

#ifdef __cplusplus
}
#endif

#endif /* FERMIX_B200_XLA_H */
