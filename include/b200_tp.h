/*
 * b200_tp.h — head-sharded tensor parallelism for the attention block: the communicator
 * and the cross-GPU sum of the `to_out` partials.
 *
 * Under head sharding GPU g owns heads [g*H/N, (g+1)*H/N): its attention output
 * [T, (H/N)*D] times its rows of W_out gives a full-width partial [T, 4096] that must be
 * summed over the N GPUs once per block (the all-reduce after `to_out`,
 * src/transformer.rs:196 under the sharding the reference's service describes).  These
 * entry points wrap NCCL so a host in any language can set up the group and issue the sum
 * on its own stream; the fused alternative (the reduction inside the `to_out` GEMM's
 * epilogue over NVLink peer memory) is b200_gemm_scatter + b200_reduce_gather_bf16 in
 * b200_gemm.h.
 *
 * NCCL is loaded at run time ("libnccl.so.2"; the copy already in the process when there
 * is one), so the library has no link-time NCCL dependency.  Every wait on the group is
 * bounded by the communicator's timeout: a peer that never joins, or dies, ends the call
 * with B200_ERR_DEVICE_TIMEOUT and the communicator is aborted (it must still be
 * destroyed).  Return codes are the b200_status values of b200_attn.h.
 */
#ifndef B200_TP_H_
#define B200_TP_H_

#include <stddef.h>
#include <stdint.h>

#include "b200_attn.h"

#ifdef __cplusplus
extern "C" {
#endif

#define B200_TP_ID_BYTES 128 /* size of ncclUniqueId */

typedef struct b200_tp_comm b200_tp_comm; /* opaque */

/* b200_dtype (B200_DTYPE_BF16 / B200_DTYPE_F32 here) is declared in b200_attn.h. */

/* A new group id, made on one rank and handed to every rank by the caller (store, MPI,
 * file ...).  B200_ERR_UNSUPPORTED when NCCL cannot be loaded. */
int b200_tp_unique_id(uint8_t id[B200_TP_ID_BYTES]);

/* Joins rank `rank` of `nranks` to the group `id` on the current CUDA device (collective:
 * every rank calls it).  The join, and every later wait of b200_tp_wait, gives up after
 * timeout_ms (0 = 60 000). */
int b200_tp_init(b200_tp_comm** comm, const uint8_t id[B200_TP_ID_BYTES], int32_t nranks,
                 int32_t rank, uint32_t timeout_ms);

/* Wraps a communicator the caller already has (an ncclComm_t, e.g. the host framework's
 * own); it is not destroyed by b200_tp_destroy. */
int b200_tp_init_from_nccl(b200_tp_comm** comm, void* nccl_comm, uint32_t timeout_ms);

int b200_tp_rank(const b200_tp_comm* comm);
int b200_tp_size(const b200_tp_comm* comm);

/* In-place sum over the group of `partial` (device, n elements of `dtype`), enqueued on
 * `stream` and ordered with the caller's work there; no host sync.  Replaces the
 * per-block all-reduce of the `to_out` partials (ncclAllReduce(sum)). */
int b200_tp_out_proj_allreduce(b200_tp_comm* comm, void* partial, size_t n, int32_t dtype,
                               b200_stream_t stream);

/* Host wait until the work enqueued on `stream` is done, bounded by the communicator's
 * timeout and watching NCCL's asynchronous error.  B200_ERR_DEVICE_TIMEOUT (timeout) or
 * B200_ERR_CUDA (NCCL or CUDA error) abort a communicator made by b200_tp_init; one given
 * to b200_tp_init_from_nccl is left to its owner.  Either way the handle refuses further
 * collectives. */
int b200_tp_wait(b200_tp_comm* comm, b200_stream_t stream);

/* Frees the communicator (aborting it first when a wait failed). */
int b200_tp_destroy(b200_tp_comm* comm);

#ifdef __cplusplus
}
#endif

#endif /* B200_TP_H_ */
