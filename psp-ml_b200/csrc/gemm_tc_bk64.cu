// gemm_tc_bk64.cu - the tcgen05 GEMM kernels with 64-byte K blocks.
#include "gemm_tc.cuh"

namespace pspml {
namespace tcg {

template cudaError_t run_tc_bn<64>(int, int, const CUtensorMap&, const CUtensorMap&,
                                   const TcGemmArgs&, const EpiTable*, int, cudaStream_t);

}  // namespace tcg
}  // namespace pspml
