// libpkt_b200's own instantiation of the persistent megakernel
// (include/pk/detail/megakernel.cuh): the built-in opcodes only.
#include "../../include/pk/detail/megakernel.cuh"

namespace pkb {

cudaError_t max_resident_blocks(int pair, int* blocks) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  return pair == 2 ? prepare_variant<2>(dev, blocks) : prepare_variant<1>(dev, blocks);
}

cudaError_t launch_megakernel(const KParams& p, int blocks, cudaStream_t stream, int pair) {
  if (pair == 2) return launch_variant<2>(p, blocks, stream);
  return launch_variant<1>(p, blocks, stream);
}

}  // namespace pkb
