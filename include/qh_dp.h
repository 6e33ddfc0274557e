/* SPDX-License-Identifier: MIT
 *
 * qh_dp.h -- data parallelism over independent sequences: one process per
 * GPU, weights replicated, no per-layer collective; after each decode step
 * the sampled tokens of every rank are gathered over NCCL (NVLink /
 * NVSwitch within a node). No counterpart in the reference, which runs one
 * process on the CPU; this is the token exchange of the multi-GPU batched
 * decode (64 sequences per GPU).
 *
 * Set-up: rank 0 calls qh_dp_unique_id and hands the QH_DP_ID_BYTES bytes
 * to every rank by any channel (a launcher's store, a file, a socket); each
 * rank then calls qh_dp_create with its device current. NCCL is loaded at
 * that point (libnccl.so.2: the copy already in the process if there is
 * one); QH_ERR_UNSUPPORTED without it.
 *
 * Every rank makes the same calls in the same order. Calls are
 * asynchronous on `stream` (a cudaStream_t; NULL = the legacy default
 * stream) except qh_dp_max_f64, which synchronizes it. A rank that has left
 * makes the others' next collective fail after timeout_ms (NCCL's blocking
 * wait is replaced by a bounded poll that aborts the communicator), with
 * QH_ERR_DEVICE; the communicator is unusable afterwards.
 */
#ifndef QH_DP_H
#define QH_DP_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QH_DP_ID_BYTES 128

typedef struct qh_dp qh_dp;

/* A new unique id (rank 0), QH_DP_ID_BYTES bytes into id_out. */
int qh_dp_unique_id(void *id_out);

/* Joins the communicator of n_ranks ranks named by id as `rank`, on the
 * current CUDA device. timeout_ms bounds every later wait (0: 120000);
 * joining itself waits at most max(timeout_ms, 60000). */
int qh_dp_create(const void *id, int32_t n_ranks, int32_t rank, int32_t timeout_ms, qh_dp **out);
int qh_dp_destroy(qh_dp *dp);
int32_t qh_dp_rank(const qh_dp *dp);
int32_t qh_dp_size(const qh_dp *dp);

/* d_all[r * n + i] = rank r's d_local[i] (int32, device memory), for the
 * n tokens each rank sampled (e.g. qh_slm_device_next). Ordered on
 * `stream` after the work before it (qh_slm_advance on qh_slm_stream). */
int qh_dp_gather_tokens(qh_dp *dp, const int32_t *d_local, int32_t n, int32_t *d_all, void *stream);

/* Waits until everything queued on `stream` has finished, at most the
 * communicator's timeout (a collective a departed rank never joins ends
 * the wait with QH_ERR_DEVICE and aborts the communicator), where a plain
 * stream synchronization would wait for good. */
int qh_dp_wait(qh_dp *dp, void *stream);

/* values[i] = the maximum of values[i] over all ranks (host doubles; the
 * job's time is its slowest rank's). Synchronous. */
int qh_dp_max_f64(qh_dp *dp, double *values, int32_t n);

#ifdef __cplusplus
}
#endif

#endif /* QH_DP_H */
