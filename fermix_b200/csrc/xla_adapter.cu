// Legacy XLA custom-call adapter (include/fermix_b200_xla.h): host code only. It unpacks
// the descriptor and XLA's buffer array and calls the C entry points on XLA's stream.
#include <atomic>
#include <cstring>

#include "fermix_b200.h"
#include "fermix_b200_xla.h"

static_assert(sizeof(fermix_xla_descriptor) == 48, "the descriptor is 48 packed bytes");

namespace {

std::atomic<int> g_last_error{0};

void record(int code) {
  int zero = 0;
  if (code) g_last_error.compare_exchange_strong(zero, code);
}

// FX_ERR_SHAPE for a descriptor that is short, of another version or carries bad fields.
int parse(const char* opaque, size_t len, fermix_xla_descriptor& d) {
  if (!opaque) return FX_ERR_NULL;
  if (len != sizeof(d)) return FX_ERR_SHAPE;
  std::memcpy(&d, opaque, sizeof(d));
  if (d.magic != FX_XLA_MAGIC || d.version != FX_XLA_VERSION) return FX_ERR_SHAPE;
  if (d.op < FX_XLA_SLOGDET || d.op > FX_XLA_SLOGPF_GRAD) return FX_ERR_SHAPE;
  if (d.flags & ~31u) return FX_ERR_SHAPE;
  return FX_OK;
}

int dispatch(void* stream, void** buf, const fermix_xla_descriptor& d) {
  if (!buf) return FX_ERR_NULL;
  const bool grad = d.op == FX_XLA_SLOGDET_GRAD || d.op == FX_XLA_SLOGPF_GRAD;
  int i = 0;
  const void* a = buf[i++];
  const void* coef = (grad && (d.flags & FX_XLA_COEF)) ? buf[i++] : nullptr;
  void* sign = buf[i++];
  void* logabs = buf[i++];
  void* value = (d.flags & FX_XLA_VALUE) ? buf[i++] : nullptr;
  void* g = grad ? buf[i++] : nullptr;
  void* ws = d.workspace_bytes ? buf[i++] : nullptr;
  const size_t wsb = (size_t)d.workspace_bytes;
  const int skew = (d.flags & FX_XLA_SKEW) ? 1 : 0;
  const int conj = (d.flags & FX_XLA_CONJ_OUT) ? 1 : 0;
  const int adj = (d.flags & FX_XLA_ADJUGATE) ? 1 : 0;
  switch (d.op) {
    case FX_XLA_SLOGDET:
      return fermix_slogdet(stream, d.dtype, d.prec, d.batch, d.n, a, sign, logabs, value, ws, wsb);
    case FX_XLA_SLOGDET_GRAD:
      return fermix_slogdet_grad(stream, d.dtype, d.prec, d.batch, d.n, a, coef, conj, adj, sign, logabs, value, g,
                                 ws, wsb);
    case FX_XLA_SLOGPF:
      return fermix_slogpf(stream, d.dtype, d.prec, d.batch, d.n, skew, a, sign, logabs, value, ws, wsb);
    default:
      return fermix_slogpf_grad(stream, d.dtype, d.prec, d.batch, d.n, skew, a, coef, conj, adj, sign, logabs, value,
                                g, ws, wsb);
  }
}

}  // namespace

extern "C" {

void fermix_xla_custom_call(void* stream, void** buffers, const char* opaque, size_t opaque_len) {
  fermix_xla_descriptor d;
  int e = parse(opaque, opaque_len, d);
  if (!e) e = dispatch(stream, buffers, d);
  record(e);
}

int fermix_xla_last_error(int clear) { return clear ? g_last_error.exchange(0) : g_last_error.load(); }

}  // extern "C"
