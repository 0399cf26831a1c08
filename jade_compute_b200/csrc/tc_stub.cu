// Placeholder for the tcgen05 kernels while they are brought up.
#include "internal.hpp"
namespace jade {
bool gemm_tc_supports(const Spec &, std::string &why) { why = "tcgen05 GEMM not built"; return false; }
LaunchFn make_gemm_tc(Context *, const Spec &, std::string &) { throw IrError("tcgen05 GEMM not built"); }
LaunchFn make_attention_tc(Context *, const Spec &, std::string &) { throw IrError("tcgen05 attention not built"); }
}
