// Tensor parallelism of the model step (placeholder until the NCCL backend is wired in).
#include "model.h"

namespace q4b {

int Model::tp_allreduce_add(int, cudaStream_t) {
  return set_error(Q4B_EUNSUPPORTED, "model: tensor parallelism needs q4b_model_attach_nccl");
}
int Model::tp_finish_argmax(int32_t*, cudaStream_t) {
  return set_error(Q4B_EUNSUPPORTED, "model: tensor parallelism needs q4b_model_attach_nccl");
}

}  // namespace q4b
