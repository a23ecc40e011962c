// qz_gemm.cu -- tcgen05 Gram and output-error GEMMs (placeholder entry points
// until the tensor-core kernels land: they report QZ_ERR_UNSUPPORTED).
#include "../../include/qwantize_b200.h"
#include "qz_kernels.h"

namespace qz { int fail(int code, const char* fmt, ...); }

extern "C" int qz_gram(const uint16_t*, int64_t, int64_t, int, int, int, float*, void*) {
  return qz::fail(QZ_ERR_UNSUPPORTED, "qz_gram: not built yet");
}
extern "C" int qz_output_error_sums(const uint16_t*, int64_t, int64_t, const uint16_t*,
                                    const uint16_t*, int64_t, double*, void*) {
  return qz::fail(QZ_ERR_UNSUPPORTED, "qz_output_error_sums: not built yet");
}
