/*
 * fake_nccl.c -- a stand-in for libnccl.so.2 for the CPU tests of
 * pkv_comm.c (loaded through PKV_NCCL_LIBRARY).  TEST ONLY: it moves no
 * data and touches no GPU.
 *
 * Joining is simulated with files: ncclCommInitRankConfig creates
 * $FAKE_NCCL_DIR/<id>.<rank> and returns ncclInProgress (non-blocking mode);
 * ncclCommGetAsyncError reports ncclSuccess once all ranks' files exist, so a
 * rank that never calls init keeps the others "in progress".  Abort,
 * destroy and all-gather calls are appended to $FAKE_NCCL_DIR/log as
 * "<call> rank <r>" lines, and so is the blocking flag seen at init.
 */
#include <dirent.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

#include <nccl.h>

struct ncclComm {
    int nranks, rank;
    int blocking;
    char name[48];
};

static const char *dir_of(void) {
    const char *d = getenv("FAKE_NCCL_DIR");
    return d != NULL ? d : "/tmp";
}

static void log_line(const char *what, int rank) {
    char path[512];
    snprintf(path, sizeof path, "%s/log", dir_of());
    FILE *f = fopen(path, "a");
    if (f == NULL) return;
    fprintf(f, "%s rank %d\n", what, rank);
    fclose(f);
}

ncclResult_t ncclGetUniqueId(ncclUniqueId *id) {
    memset(id, 0, sizeof *id);
    snprintf(id->internal, sizeof id->internal, "fake%ld_%d", (long)time(NULL), (int)getpid());
    return ncclSuccess;
}

ncclResult_t ncclCommInitRankConfig(ncclComm_t *comm, int nranks, ncclUniqueId id, int rank,
                                    ncclConfig_t *config) {
    struct ncclComm *c = calloc(1, sizeof *c);
    if (c == NULL) return ncclSystemError;
    c->nranks = nranks;
    c->rank = rank;
    c->blocking = !(config != NULL && config->blocking == 0);
    snprintf(c->name, sizeof c->name, "%.32s", id.internal);
    char path[512];
    snprintf(path, sizeof path, "%s/%s.%d", dir_of(), c->name, rank);
    FILE *f = fopen(path, "w");
    if (f != NULL) fclose(f);
    log_line(c->blocking ? "init blocking" : "init nonblocking", rank);
    *comm = c;
    return c->blocking ? ncclSuccess : ncclInProgress;
}

ncclResult_t ncclCommGetAsyncError(ncclComm_t comm, ncclResult_t *state) {
    int joined = 0;
    for (int r = 0; r < comm->nranks; ++r) {
        char path[512];
        snprintf(path, sizeof path, "%s/%s.%d", dir_of(), comm->name, r);
        joined += access(path, F_OK) == 0;
    }
    *state = joined == comm->nranks ? ncclSuccess : ncclInProgress;
    return ncclSuccess;
}

ncclResult_t ncclCommAbort(ncclComm_t comm) {
    log_line("abort", comm->rank);
    free(comm);
    return ncclSuccess;
}

ncclResult_t ncclCommFinalize(ncclComm_t comm) {
    log_line("finalize", comm->rank);
    return ncclSuccess;
}

ncclResult_t ncclCommDestroy(ncclComm_t comm) {
    log_line("destroy", comm->rank);
    free(comm);
    return ncclSuccess;
}

ncclResult_t ncclAllGather(const void *send, void *recv, size_t count, ncclDataType_t type,
                           ncclComm_t comm, cudaStream_t stream) {
    (void)send; (void)recv; (void)count; (void)type; (void)stream;
    log_line("allgather", comm->rank);
    return ncclSuccess;
}

const char *ncclGetErrorString(ncclResult_t result) {
    (void)result;
    return "fake NCCL error";
}
