// SPDX-License-Identifier: MIT
//
// qh_dp.c -- the token exchange of data-parallel decoding (include/qh_dp.h)
// over NCCL. libnccl.so.2 is opened at qh_dp_create (the copy already in the
// process when a framework loaded one, else the system's), so the library
// itself loads and runs single-GPU work without NCCL. Communicators are
// non-blocking: every wait is a bounded poll of ncclCommGetAsyncError and the
// stream, and a wait that runs out aborts the communicator and returns
// QH_ERR_DEVICE instead of hanging on a rank that has left.

#define _POSIX_C_SOURCE 200809L

#include <dlfcn.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <cuda_runtime_api.h>
#include <nccl.h>

#include "qh_backend.h"
#include "qh_dp.h"

_Static_assert(sizeof(ncclUniqueId) == QH_DP_ID_BYTES, "ncclUniqueId size");

// qh_last_error() message of the calling thread (qh_api.cu)
void qh_internal_set_error(const char *msg);

// Joining takes the peers' bootstrap and the transport set-up: at least a
// minute, whatever the communicator's own timeout.
#define QH_DP_CREATE_MIN_MS 60000

static int dp_fail(int code, const char *msg) {
    qh_internal_set_error(msg);
    return code;
}

static struct {
    int loaded;
    ncclResult_t (*get_unique_id)(ncclUniqueId *);
    ncclResult_t (*init_rank_config)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *);
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*async_error)(ncclComm_t, ncclResult_t *);
    ncclResult_t (*abort_comm)(ncclComm_t);
    ncclResult_t (*destroy)(ncclComm_t);
} N;

struct qh_dp {
    ncclComm_t comm;
    int32_t rank, size, timeout_ms, dead;
    int device;
    double *d_vals;
    int32_t cap_vals;
};

static int load_nccl(void) {
    if (N.loaded) return N.loaded > 0 ? QH_OK : QH_ERR_UNSUPPORTED;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    N.loaded = -1;
    if (!h) return dp_fail(QH_ERR_UNSUPPORTED, "qh_dp: libnccl.so.2 not found");
#define SYM(f, name) *(void **)&N.f = dlsym(h, name); if (!N.f) return QH_ERR_UNSUPPORTED;
    SYM(get_unique_id, "ncclGetUniqueId")
    SYM(init_rank_config, "ncclCommInitRankConfig")
    SYM(all_gather, "ncclAllGather")
    SYM(all_reduce, "ncclAllReduce")
    SYM(async_error, "ncclCommGetAsyncError")
    SYM(abort_comm, "ncclCommAbort")
    SYM(destroy, "ncclCommDestroy")
#undef SYM
    N.loaded = 1;
    return QH_OK;
}

static double now_ms(void) {
    struct timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return 1e3 * (double)t.tv_sec + 1e-6 * (double)t.tv_nsec;
}

static void nap(void) {
    struct timespec t = {0, 20000};  // 20 us
    nanosleep(&t, NULL);
}

// Waits (bounded) until the communicator has no operation in progress on
// the host side; aborts it on an error or a timeout.
static int settle(qh_dp *dp, int32_t limit_ms) {
    const double t0 = now_ms();
    ncclResult_t st = ncclSuccess;
    for (;;) {
        if (N.async_error(dp->comm, &st) != ncclSuccess) st = ncclSystemError;
        if (st == ncclSuccess) return QH_OK;
        if (st != ncclInProgress || now_ms() - t0 > limit_ms) break;
        nap();
    }
    N.abort_comm(dp->comm);
    dp->dead = 1;
    return dp_fail(QH_ERR_DEVICE, st == ncclInProgress ? "qh_dp: a collective did not complete within the timeout"
                                                        : "qh_dp: NCCL reported an error");
}

// Waits (bounded) until every operation queued on the stream has finished.
static int wait_stream(qh_dp *dp, cudaStream_t s) {
    const double t0 = now_ms();
    for (;;) {
        const cudaError_t e = cudaStreamQuery(s);
        if (e == cudaSuccess) return QH_OK;
        if (e != cudaErrorNotReady) return QH_ERR_CUDA;
        ncclResult_t st = ncclSuccess;
        N.async_error(dp->comm, &st);
        if ((st != ncclSuccess && st != ncclInProgress) || now_ms() - t0 > dp->timeout_ms) break;
        nap();
    }
    N.abort_comm(dp->comm);
    dp->dead = 1;
    return dp_fail(QH_ERR_DEVICE, "qh_dp: the stream's work did not complete within the timeout (a rank left?)");
}

int qh_dp_unique_id(void *id_out) {
    if (!id_out) return QH_ERR_INVALID;
    int rc = load_nccl();
    if (rc) return rc;
    ncclUniqueId id;
    if (N.get_unique_id(&id) != ncclSuccess) return QH_ERR_DEVICE;
    memcpy(id_out, &id, sizeof(id));
    return QH_OK;
}

int qh_dp_create(const void *id, int32_t n_ranks, int32_t rank, int32_t timeout_ms, qh_dp **out) {
    if (!id || !out || n_ranks < 1 || rank < 0 || rank >= n_ranks || timeout_ms < 0) return QH_ERR_INVALID;
    *out = NULL;
    int rc = load_nccl();
    if (rc) return rc;
    qh_dp *dp = (qh_dp *)calloc(1, sizeof(*dp));
    if (!dp) return QH_ERR_INVALID;
    dp->rank = rank;
    dp->size = n_ranks;
    dp->timeout_ms = timeout_ms ? timeout_ms : 120000;
    if (cudaGetDevice(&dp->device) != cudaSuccess) {
        free(dp);
        return QH_ERR_CUDA;
    }
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = N.init_rank_config(&dp->comm, n_ranks, uid, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        free(dp);
        return dp_fail(QH_ERR_DEVICE, "qh_dp: ncclCommInitRankConfig failed");
    }
    rc = settle(dp, dp->timeout_ms > QH_DP_CREATE_MIN_MS ? dp->timeout_ms : QH_DP_CREATE_MIN_MS);
    if (rc) {
        free(dp);
        return rc;
    }
    *out = dp;
    return QH_OK;
}

int qh_dp_destroy(qh_dp *dp) {
    if (!dp) return QH_OK;
    if (!dp->dead) {
        N.destroy(dp->comm);
    }
    if (dp->d_vals) qh_free(dp->d_vals);
    free(dp);
    return QH_OK;
}

int32_t qh_dp_rank(const qh_dp *dp) { return dp ? dp->rank : -1; }
int32_t qh_dp_size(const qh_dp *dp) { return dp ? dp->size : -1; }

int qh_dp_gather_tokens(qh_dp *dp, const int32_t *d_local, int32_t n, int32_t *d_all, void *stream) {
    if (!dp || !d_local || !d_all || n <= 0) return QH_ERR_INVALID;
    if (dp->dead) return QH_ERR_DEVICE;
    const ncclResult_t r = N.all_gather(d_local, d_all, (size_t)n, ncclInt32, dp->comm, (cudaStream_t)stream);
    if (r != ncclSuccess && r != ncclInProgress) return dp_fail(QH_ERR_DEVICE, "qh_dp: ncclAllGather failed");
    return settle(dp, dp->timeout_ms);
}

int qh_dp_wait(qh_dp *dp, void *stream) {
    if (!dp) return QH_ERR_INVALID;
    if (dp->dead) return QH_ERR_DEVICE;
    return wait_stream(dp, (cudaStream_t)stream);
}

int qh_dp_max_f64(qh_dp *dp, double *values, int32_t n) {
    if (!dp || !values || n <= 0) return QH_ERR_INVALID;
    if (dp->dead) return QH_ERR_DEVICE;
    if (n > dp->cap_vals) {
        if (dp->d_vals) qh_free(dp->d_vals);
        dp->d_vals = NULL;
        dp->cap_vals = 0;
        if (qh_malloc((void **)&dp->d_vals, sizeof(double) * (size_t)n)) return QH_ERR_CUDA;
        dp->cap_vals = n;
    }
    cudaStream_t s = NULL;
    int rc = qh_memcpy_h2d(dp->d_vals, values, sizeof(double) * (size_t)n, s);
    if (rc) return rc;
    const ncclResult_t r = N.all_reduce(dp->d_vals, dp->d_vals, (size_t)n, ncclFloat64, ncclMax, dp->comm, s);
    if (r != ncclSuccess && r != ncclInProgress) return dp_fail(QH_ERR_DEVICE, "qh_dp: ncclAllReduce failed");
    rc = settle(dp, dp->timeout_ms);
    if (!rc) rc = wait_stream(dp, s);
    if (!rc) rc = qh_memcpy_d2h(values, dp->d_vals, sizeof(double) * (size_t)n, s);
    if (!rc) rc = qh_stream_sync(s);
    return rc;
}
