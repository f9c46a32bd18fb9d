#include "chunk_layout.cuh"
namespace gdn2 {
int chunk_bwd_launch(const gdn2_chunk_args&, const gdn2_chunk_grads&, const ChunkWs&, const BwdWs&, cudaStream_t) {
  return GDN2_ERR_FLAGS;
}
}
