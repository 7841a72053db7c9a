// Tensor parallelism of the model step over NCCL (one process per GPU, NVLink/NVSwitch).
//
// Shards (made by the caller, see q4b.llama): wqkv rows of this rank's q/k/v heads, wgu rows of its
// slice of the intermediate size (gate | up kept per rank), wo and wdown columns of the matching
// K slices, lm_head rows [r V/t, (r+1) V/t) of the full embedding table. Per layer the wo and wdown
// partial outputs are all-reduced (sum, fp32) and added to the replicated residual stream; the
// greedy head gathers every rank's (value, index) key and keeps the largest value, lowest index on
// ties (torch.argmax's first maximum). NCCL is loaded at run time, so libq4b.so needs it only for
// tensor parallelism; the calls are captured in the runner's CUDA graphs like the kernels.
#include <dlfcn.h>
#include <nccl.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <vector>

#include "model.h"

namespace q4b {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
};

static const NcclApi* nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      const char* p = std::getenv("Q4B_NCCL_LIB");
      if (p) h = dlopen(p, RTLD_NOW | RTLD_GLOBAL);
    }
    if (!h) return;
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_reduce && api.all_gather &&
             api.error_string;
  });
  return api.ok ? &api : nullptr;
}

static int nccl_err(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return Q4B_OK;
  return set_error(Q4B_ECUDA, "%s: NCCL error %d (%s)", what, (int)r, nccl() ? nccl()->error_string(r) : "?");
}

// h += y over n elements (the all-reduced partial of a row-split projection)
__global__ void residual_add_kernel(float* __restrict__ h, const float* __restrict__ y, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) h[i] += y[i];
}

// the largest gathered key wins; publish its token and clear the accumulator for the next step
__global__ void argmax_gather_kernel(DecodeState* st, const unsigned long long* keys, int n, int32_t* token_log) {
  if (threadIdx.x != 0) return;
  unsigned long long best = 0;
  for (int i = 0; i < n; ++i) best = max(best, keys[i]);
  st->best = 0ull;
  publish_token(st, token_log, (int32_t)argmax_index(best));
}

int Model::tp_allreduce_add(int C, cudaStream_t st) {
  if (!comm) return set_error(Q4B_ESTATE, "model: tensor parallelism needs q4b_model_attach_tp");
  int rc = nccl_err(nccl()->all_reduce(y, y, (size_t)C * D, ncclFloat, ncclSum, reinterpret_cast<ncclComm_t>(comm), st),
                    "allreduce");
  if (rc) return rc;
  const int n = C * D;
  residual_add_kernel<<<(n + 255) / 256, 256, 0, st>>>(h, y, n);
  return check_launch("residual_add");
}

int Model::tp_finish_argmax(int32_t* token_log, cudaStream_t st) {
  if (!comm) return set_error(Q4B_ESTATE, "model: tensor parallelism needs q4b_model_attach_tp");
  int rc = nccl_err(nccl()->all_gather(&state->best, gather, 1, ncclUint64, reinterpret_cast<ncclComm_t>(comm), st),
                    "allgather");
  if (rc) return rc;
  argmax_gather_kernel<<<1, 32, 0, st>>>(state, gather, cfg.tp_size, token_log);
  return check_launch("argmax_gather");
}

// Maps every rank's `local` allocation (a cudaMalloc base pointer of the same size on each rank)
// into this process: the IPC handles are all-gathered over the communicator, every peer's handle is
// opened with peer access, and peers[rank] receives each rank's mapped pointer (peers[own rank] is
// left as the caller set it). Collective: every rank calls it in the same order.
int Model::tp_map_peers(void* local, void** peers) {
  if (!comm) return set_error(Q4B_ESTATE, "model: tensor parallelism needs q4b_model_attach_tp");
  const int t = cfg.tp_size;
  cudaIpcMemHandle_t own;
  cudaError_t e = cudaIpcGetMemHandle(&own, local);
  if (e != cudaSuccess) return set_error(Q4B_ECUDA, "tp_map_peers: cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  std::vector<cudaIpcMemHandle_t> all(t);
  unsigned char* dbuf = nullptr;
  cudaStream_t st = nullptr;
  e = cudaMalloc(&dbuf, sizeof(cudaIpcMemHandle_t) * (t + 1));
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMemcpy(dbuf, &own, sizeof(own), cudaMemcpyHostToDevice);
  int rc = Q4B_OK;
  if (e != cudaSuccess) {
    rc = set_error(Q4B_ECUDA, "tp_map_peers: staging: %s", cudaGetErrorString(e));
  } else {
    rc = nccl_err(nccl()->all_gather(dbuf, dbuf + sizeof(own), sizeof(own), ncclUint8,
                                     reinterpret_cast<ncclComm_t>(comm), st),
                  "allgather(ipc handles)");
    if (!rc) e = cudaStreamSynchronize(st);
    if (!rc && e == cudaSuccess) e = cudaMemcpy(all.data(), dbuf + sizeof(own), sizeof(own) * t, cudaMemcpyDeviceToHost);
    if (!rc && e != cudaSuccess) rc = set_error(Q4B_ECUDA, "tp_map_peers: gather: %s", cudaGetErrorString(e));
  }
  if (st) cudaStreamDestroy(st);
  if (dbuf) cudaFree(dbuf);
  for (int r = 0; r < t && !rc; ++r) {
    if (r == cfg.tp_rank) continue;
    void* p = nullptr;
    e = cudaIpcOpenMemHandle(&p, all[r], cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      rc = set_error(Q4B_ECUDA, "tp_map_peers: cudaIpcOpenMemHandle(rank %d): %s", r, cudaGetErrorString(e));
      break;
    }
    mk_mapped.push_back(p);
    peers[r] = p;
  }
  return rc;
}

void Model::tp_release() {
  for (void* p : mk_mapped) cudaIpcCloseMemHandle(p);
  mk_mapped.clear();
  mk_peer_h.clear();
  mk_peer_sync.clear();
  mk_ready = false;
  if (comm && nccl()) nccl()->comm_destroy(reinterpret_cast<ncclComm_t>(comm));
  comm = nullptr;
}

}  // namespace q4b

using namespace q4b;

extern "C" int q4b_tp_unique_id(unsigned char* id, int id_bytes) {
  if (!id || id_bytes < (int)sizeof(ncclUniqueId)) return set_error(Q4B_EINVAL, "tp_unique_id: need %zu bytes",
                                                                   sizeof(ncclUniqueId));
  const NcclApi* api = nccl();
  if (!api) return set_error(Q4B_EUNSUPPORTED, "tp_unique_id: libnccl.so.2 not found (set Q4B_NCCL_LIB)");
  ncclUniqueId u;
  int rc = nccl_err(api->get_unique_id(&u), "ncclGetUniqueId");
  if (rc) return rc;
  memcpy(id, &u, sizeof(u));
  return Q4B_OK;
}

extern "C" int q4b_model_attach_tp(q4b_model* model, const unsigned char* id, int id_bytes) {
  Model* m = reinterpret_cast<Model*>(model);
  if (!m || !id || id_bytes < (int)sizeof(ncclUniqueId)) return set_error(Q4B_EINVAL, "model_attach_tp: bad argument");
  if (m->cfg.tp_size < 2) return set_error(Q4B_EINVAL, "model_attach_tp: the model was created with tp_size 1");
  const NcclApi* api = nccl();
  if (!api) return set_error(Q4B_EUNSUPPORTED, "model_attach_tp: libnccl.so.2 not found (set Q4B_NCCL_LIB)");
  m->tp_release();
  ncclUniqueId u;
  memcpy(&u, id, sizeof(u));
  ncclComm_t c = nullptr;
  int rc = nccl_err(api->comm_init_rank(&c, m->cfg.tp_size, u, m->cfg.tp_rank), "ncclCommInitRank");
  if (rc) return rc;
  m->comm = reinterpret_cast<ncclComm*>(c);
  if (!m->gather && (rc = m->alloc((void**)&m->gather, sizeof(unsigned long long) * m->cfg.tp_size, true))) return rc;
  return Q4B_OK;
}

// ---- standalone collectives (tensor-parallel callers outside the model) ---------------------------

struct q4b_tp {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
};

namespace q4b {
// token = index of the largest of n gathered keys (lowest index on equal values)
__global__ void keys_max_kernel(const unsigned long long* keys, int n, int32_t* token) {
  if (threadIdx.x != 0) return;
  unsigned long long best = 0ull;
  for (int i = 0; i < n; ++i) best = max(best, keys[i]);
  *token = (int32_t)argmax_index(best);
}
}  // namespace q4b

extern "C" int q4b_tp_init(int rank, int world, const unsigned char* id, int id_bytes, q4b_tp** out) {
  if (!out || !id || id_bytes < (int)sizeof(ncclUniqueId) || world < 1 || rank < 0 || rank >= world)
    return set_error(Q4B_EINVAL, "tp_init: bad arguments");
  *out = nullptr;
  const NcclApi* api = nccl();
  if (!api) return set_error(Q4B_EUNSUPPORTED, "tp_init: libnccl.so.2 not found (set Q4B_NCCL_LIB)");
  ncclUniqueId u;
  memcpy(&u, id, sizeof(u));
  ncclComm_t c = nullptr;
  int rc = nccl_err(api->comm_init_rank(&c, world, u, rank), "ncclCommInitRank");
  if (rc) return rc;
  q4b_tp* t = new (std::nothrow) q4b_tp;
  if (!t) {
    api->comm_destroy(c);
    return set_error(Q4B_ENOMEM, "tp_init: out of host memory");
  }
  t->comm = c;
  t->rank = rank;
  t->world = world;
  *out = t;
  return Q4B_OK;
}

extern "C" void q4b_tp_destroy(q4b_tp* tp) {
  if (!tp) return;
  if (tp->comm && nccl()) nccl()->comm_destroy(tp->comm);
  delete tp;
}

static int tp_allreduce(q4b_tp* tp, void* buf, size_t n, ncclDataType_t t, const char* what, q4b_stream_t stream) {
  if (!tp || !tp->comm || (!buf && n)) return set_error(Q4B_EINVAL, "%s: bad arguments", what);
  if (!n) return Q4B_OK;
  return nccl_err(nccl()->all_reduce(buf, buf, n, t, ncclSum, tp->comm, as_stream(stream)), what);
}

extern "C" int q4b_tp_allreduce_f16(q4b_tp* tp, void* buf, size_t n, q4b_stream_t stream) {
  return tp_allreduce(tp, buf, n, ncclFloat16, "tp_allreduce_f16", stream);
}

extern "C" int q4b_tp_allreduce_f32(q4b_tp* tp, float* buf, size_t n, q4b_stream_t stream) {
  return tp_allreduce(tp, buf, n, ncclFloat32, "tp_allreduce_f32", stream);
}

extern "C" size_t q4b_tp_argmax_workspace(const q4b_tp* tp) {
  return tp ? sizeof(unsigned long long) * (size_t)(tp->world + 1) : 0;
}

extern "C" int q4b_tp_argmax_gather(q4b_tp* tp, const float* logits, int n_local, int index_offset, int32_t* token,
                                    void* workspace, size_t workspace_bytes, q4b_stream_t stream) {
  if (!tp || !tp->comm || !logits || !token || n_local < 1 || index_offset < 0)
    return set_error(Q4B_EINVAL, "tp_argmax_gather: bad arguments");
  if (!workspace || workspace_bytes < q4b_tp_argmax_workspace(tp) || !aligned(workspace, 8))
    return set_error(Q4B_EINVAL, "tp_argmax_gather: workspace of %zu bytes needed", q4b_tp_argmax_workspace(tp));
  cudaStream_t st = as_stream(stream);
  auto* keys = reinterpret_cast<unsigned long long*>(workspace);
  int rc = argmax_run(logits, n_local, index_offset, keys, nullptr, st);
  if (rc) return rc;
  rc = nccl_err(nccl()->all_gather(keys, keys + 1, 1, ncclUint64, tp->comm, st), "tp_argmax_gather allgather");
  if (rc) return rc;
  keys_max_kernel<<<1, 32, 0, st>>>(keys + 1, tp->world, token);
  return check_launch("tp_argmax_gather");
}
