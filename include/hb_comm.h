/* hummingbird-b200: C ABI of the multi-GPU exchange steps (NCCL over NVLink), built as libhb_comm.so so the
 * attention library itself does not depend on NCCL.
 *
 * The reference runs on one TPU chip and has no counterpart; these are the two exchanges its kernels admit
 * when the work is split over the GPUs of one node:
 *   - band attention sharded by sequence: each rank needs `window` rows on each side from its neighbours
 *     (band rows depend only on +-window rows, band_attention.py:15-19);
 *   - dense attention sharded by head pair: the per-rank (B, L, pairs * 128) outputs are gathered into
 *     (B, L, H * 64) before `to_out` (head pairs are independent, dense_attention.py:126-127).
 *
 * Conventions follow hb_b200.h (caller-owned device buffers, explicit stream, HbStatus return). Every call
 * that waits on other ranks takes a host-side deadline: a communicator that cannot finish initialising or
 * enqueueing in time is aborted and the call returns HB_ERR_TIMEOUT (status 6); NCCL errors are HB_ERR_NCCL
 * (8). A communicator is used from one host thread at a time.
 */
#ifndef HB_COMM_H_
#define HB_COMM_H_

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HB_COMM_ID_BYTES 128

typedef struct HbComm* hb_comm_t;

/* A new communicator id (HB_COMM_ID_BYTES bytes). One rank creates it and hands it to all the others. */
int hb_comm_unique_id(void* id_out);

/* Join communicator `id` as `rank` of `nranks` on the current CUDA device (non-blocking NCCL init polled
 * until ready; after `timeout_ms` it is aborted and HB_ERR_TIMEOUT is returned, comm set to NULL). */
int hb_comm_init(const void* id, int nranks, int rank, int timeout_ms, hb_comm_t* comm);

/* Halo exchange of a sequence-sharded band-attention input. `buf` holds, per batch element b (at
 * b * batch_stride_bytes), `before + own + after` rows of `row_bytes` bytes: the halo received from rank - 1,
 * this rank's own rows, the halo received from rank + 1. This rank sends its first `send_left` own rows to
 * rank - 1 and its last `send_right` own rows to rank + 1 (the neighbours' halo sizes). One grouped NCCL
 * send/recv on `stream`. */
int hb_comm_halo_exchange(hb_comm_t comm, void* buf, int batch, int64_t batch_stride_bytes, int64_t row_bytes,
                          int before, int own, int after, int send_left, int send_right, int timeout_ms,
                          cudaStream_t stream);

/* Gather the head-pair slices of dense attention: `local` is this rank's (rows, widths_bytes[rank]) block
 * (row stride local_row_bytes); `gathered` is scratch of nranks * rows * max(widths_bytes) bytes; `out`
 * receives (rows, sum(widths_bytes)) with rank r's columns at offset sum(widths_bytes[:r]) (row stride
 * out_row_bytes). Widths are multiples of 16 bytes (uneven pair splits allowed). */
int hb_comm_allgather_pairs(hb_comm_t comm, const void* local, int64_t local_row_bytes, int64_t rows,
                            const int64_t* widths_bytes, void* gathered, void* out, int64_t out_row_bytes,
                            int timeout_ms, cudaStream_t stream);

/* Abort (after a failure: does not wait for outstanding work) or destroy a communicator; both free it. */
int hb_comm_abort(hb_comm_t comm);
int hb_comm_destroy(hb_comm_t comm);

/* Rank count and rank of a communicator. */
int hb_comm_size(hb_comm_t comm, int* nranks, int* rank);

#ifdef __cplusplus
}
#endif

#endif /* HB_COMM_H_ */
