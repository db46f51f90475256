// NCCL exchanges of the multi-GPU paths (include/hb_comm.h): halo send/recv for sequence-sharded band
// attention and the head-pair all-gather of dense attention. Communicators are created non-blocking so a
// rank that never arrives, or an enqueue that cannot progress, is bounded by a host-side deadline and ends
// in ncclCommAbort instead of a hang.
#include <chrono>
#include <cstdint>
#include <cstring>
#include <new>
#include <thread>

#include <cuda_runtime.h>
#include <nccl.h>

#include "../../include/hb_comm.h"
#include "hb_status.h"

struct HbComm {
  ncclComm_t nccl = nullptr;
  int nranks = 0, rank = 0;
};

namespace {

static_assert(sizeof(ncclUniqueId) == HB_COMM_ID_BYTES, "NCCL unique id size");

// Poll a non-blocking communicator until its last operation left ncclInProgress; abort at the deadline.
int settle(HbComm* c, int timeout_ms) {
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
  while (true) {
    ncclResult_t state = ncclSuccess;
    if (ncclCommGetAsyncError(c->nccl, &state) != ncclSuccess) return HB_ERR_NCCL;
    if (state == ncclSuccess) return HB_OK;
    if (state != ncclInProgress) return HB_ERR_NCCL;
    if (std::chrono::steady_clock::now() > deadline) return HB_ERR_TIMEOUT;
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

int check_call(HbComm* c, ncclResult_t r, int timeout_ms) {
  if (r == ncclSuccess || r == ncclInProgress) return settle(c, timeout_ms);
  return HB_ERR_NCCL;
}

constexpr int kMaxRanks = 64;
struct PairTables {
  int64_t width[kMaxRanks], offset[kMaxRanks];
};

// out[row, offset_r + x] = gathered[r][row, x] for x < width_r: one thread per 16-byte piece.
__global__ void scatter_pairs_kernel(const uint8_t* __restrict__ gathered, int64_t rows, int64_t wmax,
                                     const __grid_constant__ PairTables t, int nranks, uint8_t* __restrict__ out,
                                     int64_t out_row_bytes) {
  const int64_t pieces_per_row = wmax / 16;
  const int64_t total = (int64_t)nranks * rows * pieces_per_row;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t piece = i % pieces_per_row;
    const int64_t rr = i / pieces_per_row;
    const int r = static_cast<int>(rr / rows);
    const int64_t row = rr - (int64_t)r * rows;
    if (piece * 16 >= t.width[r]) continue;
    const uint4 v = *reinterpret_cast<const uint4*>(gathered + ((int64_t)r * rows + row) * wmax + piece * 16);
    *reinterpret_cast<uint4*>(out + row * out_row_bytes + t.offset[r] + piece * 16) = v;
  }
}

}  // namespace

extern "C" int hb_comm_unique_id(void* id_out) {
  if (!id_out) return HB_ERR_NULL;
  ncclUniqueId id;
  if (ncclGetUniqueId(&id) != ncclSuccess) return HB_ERR_NCCL;
  std::memcpy(id_out, &id, sizeof(id));
  return HB_OK;
}

extern "C" int hb_comm_init(const void* id, int nranks, int rank, int timeout_ms, hb_comm_t* comm) {
  if (!id || !comm) return HB_ERR_NULL;
  *comm = nullptr;
  if (nranks < 1 || rank < 0 || rank >= nranks || timeout_ms < 1) return HB_ERR_SHAPE;
  HbComm* c = new (std::nothrow) HbComm;
  if (!c) return HB_ERR_LAUNCH;
  c->nranks = nranks;
  c->rank = rank;
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
  config.blocking = 0;
  const ncclResult_t r = ncclCommInitRankConfig(&c->nccl, nranks, uid, rank, &config);
  int st = (r == ncclSuccess || r == ncclInProgress) && c->nccl ? settle(c, timeout_ms) : HB_ERR_NCCL;
  if (st != HB_OK) {
    if (c->nccl) ncclCommAbort(c->nccl);
    delete c;
    return st;
  }
  *comm = c;
  return HB_OK;
}

extern "C" int hb_comm_halo_exchange(hb_comm_t comm, void* buf, int batch, int64_t batch_stride_bytes,
                                     int64_t row_bytes, int before, int own, int after, int send_left,
                                     int send_right, int timeout_ms, cudaStream_t stream) {
  if (!comm || !buf) return HB_ERR_NULL;
  if (batch < 1 || row_bytes < 1 || before < 0 || after < 0 || own < 1 || send_left < 0 || send_right < 0 ||
      send_left > own || send_right > own || timeout_ms < 1 ||
      batch_stride_bytes < (int64_t)(before + own + after) * row_bytes)
    return HB_ERR_SHAPE;
  if ((comm->rank == 0 && (before || send_left)) || (comm->rank == comm->nranks - 1 && (after || send_right)))
    return HB_ERR_SHAPE;
  uint8_t* base = static_cast<uint8_t*>(buf);
  const int left = comm->rank - 1, right = comm->rank + 1;
  if (ncclGroupStart() != ncclSuccess) return HB_ERR_NCCL;
  ncclResult_t r = ncclSuccess;
  for (int b = 0; b < batch && (r == ncclSuccess || r == ncclInProgress); ++b) {
    uint8_t* rows = base + (int64_t)b * batch_stride_bytes;
    uint8_t* own0 = rows + (int64_t)before * row_bytes;
    uint8_t* own1 = own0 + (int64_t)own * row_bytes;
    if (left >= 0 && send_left) r = ncclSend(own0, send_left * row_bytes, ncclUint8, left, comm->nccl, stream);
    if ((r == ncclSuccess || r == ncclInProgress) && left >= 0 && before)
      r = ncclRecv(rows, before * row_bytes, ncclUint8, left, comm->nccl, stream);
    if ((r == ncclSuccess || r == ncclInProgress) && right < comm->nranks && send_right)
      r = ncclSend(own1 - send_right * row_bytes, send_right * row_bytes, ncclUint8, right, comm->nccl, stream);
    if ((r == ncclSuccess || r == ncclInProgress) && right < comm->nranks && after)
      r = ncclRecv(own1, after * row_bytes, ncclUint8, right, comm->nccl, stream);
  }
  const ncclResult_t e = ncclGroupEnd();
  if (r != ncclSuccess && r != ncclInProgress) return HB_ERR_NCCL;
  return check_call(comm, e, timeout_ms);
}

extern "C" int hb_comm_allgather_pairs(hb_comm_t comm, const void* local, int64_t local_row_bytes, int64_t rows,
                                       const int64_t* widths_bytes, void* gathered, void* out, int64_t out_row_bytes,
                                       int timeout_ms, cudaStream_t stream) {
  if (!comm || !local || !widths_bytes || !gathered || !out) return HB_ERR_NULL;
  const int n = comm->nranks;
  if (rows < 1 || timeout_ms < 1 || n > kMaxRanks) return HB_ERR_SHAPE;
  PairTables t;
  int64_t wmax = 0, total = 0;
  for (int r = 0; r < n; ++r) {
    if (widths_bytes[r] < 0 || widths_bytes[r] % 16) return HB_ERR_SHAPE;
    t.width[r] = widths_bytes[r];
    t.offset[r] = total;
    total += widths_bytes[r];
    if (widths_bytes[r] > wmax) wmax = widths_bytes[r];
  }
  if (wmax == 0 || out_row_bytes < total || local_row_bytes < t.width[comm->rank]) return HB_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(gathered) | reinterpret_cast<uintptr_t>(out) | (uintptr_t)out_row_bytes) & 15u)
    return HB_ERR_ALIGN;
  // this rank's block, padded to wmax, into its slot of `gathered`, then one all-gather in place
  uint8_t* slot = static_cast<uint8_t*>(gathered) + (int64_t)comm->rank * rows * wmax;
  if (cudaMemset2DAsync(slot, wmax, 0, wmax, rows, stream) != cudaSuccess) return HB_ERR_LAUNCH;
  if (t.width[comm->rank] &&
      cudaMemcpy2DAsync(slot, wmax, local, local_row_bytes, t.width[comm->rank], rows, cudaMemcpyDeviceToDevice,
                        stream) != cudaSuccess)
    return HB_ERR_LAUNCH;
  const int st = check_call(comm, ncclAllGather(slot, gathered, rows * wmax, ncclUint8, comm->nccl, stream), timeout_ms);
  if (st != HB_OK) return st;
  const int64_t pieces = (int64_t)n * rows * (wmax / 16);
  const int grid = static_cast<int>((pieces + 255) / 256 < 4096 ? (pieces + 255) / 256 : 4096);
  scatter_pairs_kernel<<<grid, 256, 0, stream>>>(static_cast<const uint8_t*>(gathered), rows, wmax, t, n,
                                                 static_cast<uint8_t*>(out), out_row_bytes);
  return cudaGetLastError() == cudaSuccess ? HB_OK : HB_ERR_LAUNCH;
}

extern "C" int hb_comm_abort(hb_comm_t comm) {
  if (!comm) return HB_ERR_NULL;
  const ncclResult_t r = comm->nccl ? ncclCommAbort(comm->nccl) : ncclSuccess;
  delete comm;
  return r == ncclSuccess ? HB_OK : HB_ERR_NCCL;
}

extern "C" int hb_comm_destroy(hb_comm_t comm) {
  if (!comm) return HB_ERR_NULL;
  ncclResult_t r = ncclSuccess;
  if (comm->nccl) {
    r = ncclCommFinalize(comm->nccl);
    if (r == ncclSuccess || r == ncclInProgress) {
      const int st = settle(comm, 10000);
      r = st == HB_OK ? ncclCommDestroy(comm->nccl) : ncclCommAbort(comm->nccl);
    } else {
      ncclCommAbort(comm->nccl);
    }
  }
  delete comm;
  return r == ncclSuccess ? HB_OK : HB_ERR_NCCL;
}

extern "C" int hb_comm_size(hb_comm_t comm, int* nranks, int* rank) {
  if (!comm || !nranks || !rank) return HB_ERR_NULL;
  *nranks = comm->nranks;
  *rank = comm->rank;
  return HB_OK;
}
