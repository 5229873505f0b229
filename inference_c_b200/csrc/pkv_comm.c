/*
 * pkv_comm.c -- NCCL all-gather with a host deadline, for the config-4 head
 * split (each GPU decodes its KV heads, then every GPU needs every head's
 * output).
 *
 * The SDK has no multi-GPU code; its only failure handling on this path is
 * the return code and the rollback of the decode transaction
 * (src/common/attention.c:159-166).  Across GPUs a failure is a peer that
 * never joins or stops part-way, and a blocking NCCL call would then wait
 * forever.  This module therefore joins a communicator in NCCL's
 * non-blocking mode first (init returns at once and the host polls
 * ncclCommGetAsyncError against a deadline): that proves every rank is
 * alive.  The collectives then run on a second, blocking communicator
 * (initialised from its own id, in a helper thread, under the same
 * deadline): a blocking enqueue only queues work -- it never waits for
 * peers -- and is several times faster than a non-blocking one, whose
 * enqueue completes asynchronously.  Waiting for a collective polls the
 * stream and the communicator's error state against a deadline; past it,
 * ncclCommAbort ends both communicators' work (NCCL's kernels watch the
 * abort flag) and the caller gets 0 and rolls its step back.
 *
 * NCCL is loaded at run time (dlopen of PKV_NCCL_LIBRARY, default
 * libnccl.so.2 -- the one the process already has, e.g. torch's), so the
 * library has no link-time NCCL dependency and tests can substitute a fake.
 */
#define _GNU_SOURCE
#include <dlfcn.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <cuda_runtime_api.h>
#include <nccl.h>

#include "pkv_b200.h"
#include "pkv_internal.h"
#include "pkv_trace.h"

typedef struct {
    ncclResult_t (*get_unique_id)(ncclUniqueId *);
    ncclResult_t (*init_rank_config)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *);
    ncclResult_t (*get_async_error)(ncclComm_t, ncclResult_t *);
    ncclResult_t (*abort)(ncclComm_t);
    ncclResult_t (*finalize)(ncclComm_t);
    ncclResult_t (*destroy)(ncclComm_t);
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t,
                               cudaStream_t);
    const char *(*error_string)(ncclResult_t);
} NcclApi;

static NcclApi g_nccl;
static int g_nccl_ok;
static char g_nccl_why[256];
static pthread_once_t g_nccl_once = PTHREAD_ONCE_INIT;

static void load_nccl(void) {
    const char *path = getenv("PKV_NCCL_LIBRARY");
    if (path == NULL || path[0] == 0) path = "libnccl.so.2";
    void *h = dlopen(path, RTLD_NOW | RTLD_LOCAL);
    if (h == NULL) {
        snprintf(g_nccl_why, sizeof g_nccl_why, "cannot load %s: %s", path, dlerror());
        return;
    }
#define PKV_SYM(field, name)                                                          \
    *(void **)(&g_nccl.field) = dlsym(h, name);                                       \
    if (g_nccl.field == NULL) {                                                       \
        snprintf(g_nccl_why, sizeof g_nccl_why, "%s lacks %s", path, name);           \
        return;                                                                       \
    }
    PKV_SYM(get_unique_id, "ncclGetUniqueId")
    PKV_SYM(init_rank_config, "ncclCommInitRankConfig")
    PKV_SYM(get_async_error, "ncclCommGetAsyncError")
    PKV_SYM(abort, "ncclCommAbort")
    PKV_SYM(finalize, "ncclCommFinalize")
    PKV_SYM(destroy, "ncclCommDestroy")
    PKV_SYM(all_gather, "ncclAllGather")
    PKV_SYM(error_string, "ncclGetErrorString")
#undef PKV_SYM
    g_nccl_ok = 1;
}

static int nccl_ready(char *error, size_t cap, const char *what) {
    pthread_once(&g_nccl_once, load_nccl);
    if (!g_nccl_ok) pkv_internal_set_error(error, cap, "%s: %s", what, g_nccl_why);
    return g_nccl_ok;
}

struct PkvComm {
    ncclComm_t parent;  /* non-blocking: joins under a deadline */
    ncclComm_t comm;    /* blocking: the collectives */
    int device, nranks, rank;
    int aborted;
    /* completion check of the enqueued work: NULL = cudaStreamQuery(stream);
     * tests on machines without a GPU install their own */
    int (*probe)(void *arg, PkvStream stream);
    void *probe_arg;
};

static double now_s(void) {
    struct timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return (double)t.tv_sec + 1e-9 * (double)t.tv_nsec;
}

/* Between polls: spin for the first 2 ms of a wait (an enqueue or a small
 * collective settles in microseconds, and the device may be idle until the
 * host sees it), then sleep 20 us per poll. */
static void nap(double started) {
    if (now_s() - started < 2e-3) return;
    const struct timespec t = {0, 20000};
    nanosleep(&t, NULL);
}

static void abort_comm(PkvComm *c) {
    if (!c->aborted) {
        if (c->comm != NULL) (void)g_nccl.abort(c->comm);
        if (c->parent != NULL) (void)g_nccl.abort(c->parent);
        c->aborted = 1;
    }
}

/* Polls communicator `h` until its pending operation (init, split or an
 * enqueue) leaves ncclInProgress, or until `deadline`; on timeout or error
 * the communicators are aborted.  1 on success. */
static int settle(PkvComm *c, ncclComm_t h, double deadline, char *error, size_t cap,
                  const char *what, const char *waiting_for) {
    const double started = now_s();
    for (;;) {
        ncclResult_t state = ncclInProgress;
        const ncclResult_t r = g_nccl.get_async_error(h, &state);
        if (r != ncclSuccess) state = r;
        if (state == ncclSuccess) return 1;
        if (state != ncclInProgress) {
            abort_comm(c);
            pkv_internal_set_error(error, cap, "%s: NCCL error while %s: %s; communicator "
                                   "aborted", what, waiting_for, g_nccl.error_string(state));
            return 0;
        }
        if (now_s() > deadline) {
            abort_comm(c);
            pkv_internal_set_error(error, cap, "%s: timed out %s; communicator aborted", what,
                                   waiting_for);
            return 0;
        }
        nap(started);
    }
}

typedef struct {
    PkvComm *c;
    ncclUniqueId id;
    ncclResult_t result;
    int done;  /* set (atomically) when the init returned */
} BlockingInit;

static void *blocking_init_main(void *arg) {
    BlockingInit *job = (BlockingInit *)arg;
    PkvComm *c = job->c;
    if (c->device >= 0) cudaSetDevice(c->device); /* NCCL binds the current device */
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 1;
    job->result = g_nccl.init_rank_config(&c->comm, c->nranks, job->id, c->rank, &cfg);
    __atomic_store_n(&job->done, 1, __ATOMIC_RELEASE);
    return NULL;
}

/* Initialises c->comm (blocking mode) from `id` before `deadline`.  On
 * timeout the joining communicator is aborted, the helper thread is left
 * inside NCCL (it owns `c` and the job from then on) and 0 is returned; on
 * any other failure `c` is freed. */
static int init_blocking(PkvComm *c, const unsigned char *id, double deadline, char *error,
                         size_t cap, const char *what) {
    BlockingInit *job = (BlockingInit *)calloc(1, sizeof *job);
    if (job == NULL) {
        abort_comm(c);
        pkv_internal_set_error(error, cap, "%s: out of host memory", what);
        free(c);
        return 0;
    }
    job->c = c;
    memcpy(job->id.internal, id, NCCL_UNIQUE_ID_BYTES);
    pthread_t tid;
    if (pthread_create(&tid, NULL, blocking_init_main, job) != 0) {
        abort_comm(c);
        pkv_internal_set_error(error, cap, "%s: cannot start the init thread", what);
        free(job);
        free(c);
        return 0;
    }
    const double started = now_s();
    while (!__atomic_load_n(&job->done, __ATOMIC_ACQUIRE)) {
        if (now_s() > deadline) {
            pthread_detach(tid);
            if (c->parent != NULL) (void)g_nccl.abort(c->parent);
            pkv_internal_set_error(error, cap,
                                   "%s: timed out initialising the collective communicator "
                                   "(a rank stopped after joining); joining communicator "
                                   "aborted", what);
            return 0;
        }
        nap(started);
    }
    pthread_join(tid, NULL);
    const ncclResult_t r = job->result;
    free(job);
    if (r != ncclSuccess) {
        abort_comm(c);
        pkv_internal_set_error(error, cap, "%s: %s", what, g_nccl.error_string(r));
        free(c);
        return 0;
    }
    return 1;
}

int pkv_comm_unique_id(unsigned char *id, size_t id_bytes, char *error, size_t cap) {
    const char *what = "pkv_comm_unique_id";
    if (id == NULL || id_bytes != PKV_COMM_ID_BYTES) {
        pkv_internal_set_error(error, cap, "%s: needs a buffer of %d bytes", what,
                               PKV_COMM_ID_BYTES);
        return 0;
    }
    if (!nccl_ready(error, cap, what)) return 0;
    for (int k = 0; k < 2; ++k) {  /* the joining and the collectives' communicator */
        ncclUniqueId u;
        const ncclResult_t r = g_nccl.get_unique_id(&u);
        if (r != ncclSuccess) {
            pkv_internal_set_error(error, cap, "%s: %s", what, g_nccl.error_string(r));
            return 0;
        }
        memcpy(id + k * NCCL_UNIQUE_ID_BYTES, u.internal, NCCL_UNIQUE_ID_BYTES);
    }
    return 1;
}

int pkv_comm_init(const unsigned char *id, size_t id_bytes, int nranks, int rank, int device,
                  double timeout_s, PkvComm **comm, char *error, size_t cap) {
    const char *what = "pkv_comm_init";
    PKV_RANGE_PUSH(what);
    int ok = 0;
    PkvComm *c = NULL;
    if (comm != NULL) *comm = NULL;
    if (id == NULL || id_bytes != PKV_COMM_ID_BYTES || comm == NULL || nranks < 1 ||
        rank < 0 || rank >= nranks || !(timeout_s > 0)) {
        pkv_internal_set_error(error, cap, "%s: invalid arguments", what);
        goto done;
    }
    if (!nccl_ready(error, cap, what)) goto done;
    c = (PkvComm *)calloc(1, sizeof *c);
    if (c == NULL) {
        pkv_internal_set_error(error, cap, "%s: out of host memory", what);
        goto done;
    }
    c->device = device;
    c->nranks = nranks;
    c->rank = rank;
    if (device >= 0 && cudaSetDevice(device) != cudaSuccess) {
        pkv_internal_set_error(error, cap, "%s: cannot select device %d", what, device);
        goto done;
    }
    ncclUniqueId u;
    memcpy(u.internal, id, NCCL_UNIQUE_ID_BYTES);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0; /* every call returns at once; completion is polled */
    const double deadline = now_s() + timeout_s;
    ncclResult_t r = g_nccl.init_rank_config(&c->parent, nranks, u, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        pkv_internal_set_error(error, cap, "%s: %s", what, g_nccl.error_string(r));
        if (c->parent != NULL) abort_comm(c);
        goto done;
    }
    char waiting[96];
    snprintf(waiting, sizeof waiting, "after %.3g s waiting for the %d other rank(s) to join",
             timeout_s, nranks - 1);
    if (!settle(c, c->parent, deadline, error, cap, what, waiting)) goto done;
    /* the collectives' blocking communicator, initialised in a helper thread
     * (a blocking init returns only when every rank joined) under the same
     * deadline; all ranks were seen alive a moment ago */
    if (!init_blocking(c, id + NCCL_UNIQUE_ID_BYTES, deadline, error, cap, what)) {
        c = NULL;  /* owned by the helper thread if it is still inside NCCL */
        goto done;
    }
    *comm = c;
    c = NULL;
    ok = 1;
done:
    free(c);
    PKV_RANGE_POP();
    return ok;
}

int pkv_comm_all_gather(PkvComm *comm, const void *send, void *recv, size_t bytes_per_rank,
                        PkvStream stream, double timeout_s, char *error, size_t cap) {
    const char *what = "pkv_comm_all_gather";
    if (comm == NULL || send == NULL || recv == NULL || bytes_per_rank == 0 ||
        !(timeout_s > 0)) {
        pkv_internal_set_error(error, cap, "%s: invalid arguments", what);
        return 0;
    }
    if (comm->aborted) {
        pkv_internal_set_error(error, cap, "%s: the communicator was aborted", what);
        return 0;
    }
    PKV_RANGE_PUSH(what);
    const double deadline = now_s() + timeout_s;
    const ncclResult_t r = g_nccl.all_gather(send, recv, bytes_per_rank, ncclUint8, comm->comm,
                                             (cudaStream_t)stream);
    int ok;
    if (r != ncclSuccess && r != ncclInProgress) {
        abort_comm(comm);
        pkv_internal_set_error(error, cap, "%s: %s; communicator aborted", what,
                               g_nccl.error_string(r));
        ok = 0;
    } else {
        ok = settle(comm, comm->comm, deadline, error, cap, what, "enqueueing the all-gather");
    }
    PKV_RANGE_POP();
    return ok;
}

int pkv_comm_wait(PkvComm *comm, PkvStream stream, double timeout_s, char *error, size_t cap) {
    const char *what = "pkv_comm_wait";
    if (comm == NULL || !(timeout_s > 0)) {
        pkv_internal_set_error(error, cap, "%s: invalid arguments", what);
        return 0;
    }
    if (comm->aborted) {
        pkv_internal_set_error(error, cap, "%s: the communicator was aborted", what);
        return 0;
    }
    PKV_RANGE_PUSH(what);
    const double started = now_s(), deadline = started + timeout_s;
    int ok = 0;
    for (;;) {
        ncclResult_t state = ncclSuccess;
        const ncclResult_t r = comm->aborted ? ncclInvalidUsage
                                             : g_nccl.get_async_error(comm->comm, &state);
        if (r != ncclSuccess) state = r;
        if (state != ncclSuccess && state != ncclInProgress) {
            abort_comm(comm);
            pkv_internal_set_error(error, cap, "%s: NCCL error: %s; communicator aborted",
                                   what, g_nccl.error_string(state));
            break;
        }
        int done;
        if (comm->probe != NULL) {
            done = comm->probe(comm->probe_arg, stream);
        } else {
            const cudaError_t q = cudaStreamQuery((cudaStream_t)stream);
            done = q == cudaSuccess ? 1 : (q == cudaErrorNotReady ? 0 : -1);
        }
        if (done > 0) {
            ok = 1;
            break;
        }
        if (done < 0) {
            abort_comm(comm);
            pkv_internal_set_error(error, cap, "%s: the stream failed: %s; communicator aborted",
                                   what, cudaGetErrorString(cudaGetLastError()));
            break;
        }
        if (now_s() > deadline) {
            abort_comm(comm);
            pkv_internal_set_error(error, cap,
                                   "%s: the stream's work did not finish within %.3g s (a peer "
                                   "missing or stalled); communicator aborted",
                                   what, timeout_s);
            break;
        }
        nap(started);
    }
    PKV_RANGE_POP();
    return ok;
}

int pkv_comm_aborted(const PkvComm *comm) { return comm == NULL || comm->aborted; }

void pkv_comm_destroy(PkvComm *comm) {
    if (comm == NULL) return;
    if (!comm->aborted) {
        int prev = 0;
        const int have_prev = cudaGetDevice(&prev) == cudaSuccess;
        if (comm->device >= 0) cudaSetDevice(comm->device);
        /* finalize flushes outstanding work: the blocking child returns when
         * done, the non-blocking parent is polled a bounded time; whatever
         * does not settle is aborted instead of freed */
        const int child_done = g_nccl.finalize(comm->comm) == ncclSuccess;  /* blocking */
        const ncclResult_t r = child_done ? g_nccl.finalize(comm->parent) : ncclInternalError;
        const int parent_done =
            (r == ncclSuccess || r == ncclInProgress) &&
            settle(comm, comm->parent, now_s() + 10.0, NULL, 0, "pkv_comm_destroy",
                   "finalizing");
        if (child_done && parent_done) {
            (void)g_nccl.destroy(comm->comm);
            (void)g_nccl.destroy(comm->parent);
        } else {
            abort_comm(comm);
        }
        if (have_prev) cudaSetDevice(prev);
    }
    free(comm);
}

void pkv_internal_comm_set_probe(PkvComm *comm, int (*probe)(void *arg, PkvStream stream),
                                 void *arg) {
    if (comm == NULL) return;
    comm->probe = probe;
    comm->probe_arg = arg;
}
