// NCCL communicator and collectives for data-parallel training of the
// `ocl` backend.  The reference has no multi-device code at all; this is
// the gradient exchange of the data-parallel step (one process per GPU,
// NVLink / NVSwitch underneath).  Communicator set-up uses a unique id that
// the host side exchanges over torch.distributed's store.
#include <nccl.h>
#include "common.cuh"

namespace pvb2 {
static int nccl_dtype(int dt, ncclDataType_t* out) {
  switch (dt) {
    case PVB2_F32: *out = ncclFloat32; return PVB2_OK;
    case PVB2_F64: *out = ncclFloat64; return PVB2_OK;
    case PVB2_I64: *out = ncclInt64; return PVB2_OK;
    case PVB2_I32: *out = ncclInt32; return PVB2_OK;
    case PVB2_F16: *out = ncclFloat16; return PVB2_OK;
    case PVB2_BF16: *out = ncclBfloat16; return PVB2_OK;
    case PVB2_U8:
    case PVB2_BOOL: *out = ncclUint8; return PVB2_OK;
  }
  return fail(PVB2_ERR_INVALID, "nccl: unsupported dtype %d", dt);
}
}  // namespace pvb2

using namespace pvb2;

#define PVB2_NCCL_TRY(expr)                                                                               \
  do {                                                                                                    \
    ncclResult_t _r = (expr);                                                                             \
    if (_r != ncclSuccess) return fail(PVB2_ERR_NCCL, "%s failed: %s", #expr, ncclGetErrorString(_r)); \
  } while (0)

extern "C" {

int pvb2_nccl_get_unique_id(uint8_t id[PVB2_NCCL_ID_BYTES]) {
  static_assert(sizeof(ncclUniqueId) == PVB2_NCCL_ID_BYTES, "ncclUniqueId size");
  ncclUniqueId u;
  PVB2_NCCL_TRY(ncclGetUniqueId(&u));
  memcpy(id, &u, sizeof(u));
  return PVB2_OK;
}

int pvb2_nccl_comm_init(void** comm, int nranks, const uint8_t id[PVB2_NCCL_ID_BYTES], int rank) {
  ncclUniqueId u;
  memcpy(&u, id, sizeof(u));
  ncclComm_t c;
  PVB2_NCCL_TRY(ncclCommInitRank(&c, nranks, u, rank));
  *comm = c;
  return PVB2_OK;
}

int pvb2_nccl_allreduce(void* comm, const void* send, void* recv, size_t count, int dtype, int op,
                        pvb2_stream stream) {
  ncclDataType_t t;
  PVB2_TRY(nccl_dtype(dtype, &t));
  PVB2_CHECK_ARG(op == 0 || op == 1, "nccl_allreduce: op must be 0 (sum) or 1 (avg)");
  PVB2_NCCL_TRY(ncclAllReduce(send, recv, count, t, op == 0 ? ncclSum : ncclAvg, (ncclComm_t)comm, as_stream(stream)));
  return PVB2_OK;
}

int pvb2_nccl_broadcast(void* comm, void* buf, size_t count, int dtype, int root, pvb2_stream stream) {
  ncclDataType_t t;
  PVB2_TRY(nccl_dtype(dtype, &t));
  PVB2_NCCL_TRY(ncclBroadcast(buf, buf, count, t, root, (ncclComm_t)comm, as_stream(stream)));
  return PVB2_OK;
}

int pvb2_nccl_comm_destroy(void* comm) {
  if (!comm) return PVB2_OK;
  PVB2_NCCL_TRY(ncclCommDestroy((ncclComm_t)comm));
  return PVB2_OK;
}

int pvb2_nccl_comm_abort(void* comm) {
  if (!comm) return PVB2_OK;
  PVB2_NCCL_TRY(ncclCommAbort((ncclComm_t)comm));
  return PVB2_OK;
}

}  // extern "C"
