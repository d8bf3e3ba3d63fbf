/*
 * tp_nccl.c -- the collectives of the tensor-parallel engine, over NCCL
 * (NVLink / NVSwitch inside one node).  libnccl.so.2 is opened on first use,
 * so single-GPU engines and hosts without NCCL never load it; when the process
 * already has NCCL loaded (e.g. by torch.distributed) that copy is reused.
 *
 * Tensor parallelism follows the plan for the 70B configuration: column-split
 * Wq/Wk/Wv/gate/up, row-split Wo/down followed by an all-reduce(sum) of the
 * [rows, d_model] activations, vocabulary-split LM head with a gather of
 * per-rank (max, index) pairs for greedy sampling.
 */
#define _GNU_SOURCE
#include <dlfcn.h>
#include <nccl.h>
#include <pthread.h>
#include <string.h>

#include "sb_internal.h"
#include "sb_kernels.h"

static struct {
    int ok;
    ncclResult_t (*get_unique_id)(ncclUniqueId*);
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int);
    ncclResult_t (*comm_destroy)(ncclComm_t);
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t);
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                               cudaStream_t);
    const char* (*error_string)(ncclResult_t);
    ncclResult_t (*comm_split)(ncclComm_t, int, int, ncclComm_t*, ncclConfig_t*);   /* optional */
} g_nccl;
static pthread_once_t g_once = PTHREAD_ONCE_INIT;

static void nccl_open(void) {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    g_nccl.get_unique_id = dlsym(h, "ncclGetUniqueId");
    g_nccl.comm_init_rank = dlsym(h, "ncclCommInitRank");
    g_nccl.comm_destroy = dlsym(h, "ncclCommDestroy");
    g_nccl.all_reduce = dlsym(h, "ncclAllReduce");
    g_nccl.all_gather = dlsym(h, "ncclAllGather");
    g_nccl.error_string = dlsym(h, "ncclGetErrorString");
    g_nccl.comm_split = dlsym(h, "ncclCommSplit");
    g_nccl.ok = g_nccl.get_unique_id && g_nccl.comm_init_rank && g_nccl.comm_destroy &&
                g_nccl.all_reduce && g_nccl.all_gather && g_nccl.error_string;
}

static int have_nccl(void) {
    pthread_once(&g_once, nccl_open);
    if (!g_nccl.ok) sb_set_error("libnccl.so.2 not found: tensor parallelism needs NCCL");
    return g_nccl.ok;
}

static int nccl_check(ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return 0;
    sb_set_error("%s: %s", what, g_nccl.error_string(r));
    return -5;
}

int slate_cuda_tp_unique_id(void* out, size_t n) {
    if (!out || n < sizeof(ncclUniqueId)) {
        sb_set_error("tp unique id needs %zu bytes", sizeof(ncclUniqueId));
        return -1;
    }
    if (!have_nccl()) return -5;
    ncclUniqueId id;
    int rc = nccl_check(g_nccl.get_unique_id(&id), "ncclGetUniqueId");
    if (!rc) memcpy(out, &id, sizeof id);
    return rc;
}

int sb_tp_init(void** comm, int nranks, int rank, const void* id) {
    if (!have_nccl()) return -5;
    ncclUniqueId u;
    memcpy(&u, id, sizeof u);
    ncclComm_t c = NULL;
    int rc = nccl_check(g_nccl.comm_init_rank(&c, nranks, u, rank), "ncclCommInitRank");
    *comm = rc ? NULL : (void*)c;
    return rc;
}

/* A second communicator over the same ranks (ncclCommSplit with one color, a
 * collective: every rank calls it), for collectives issued on a second stream
 * beside those of the first communicator. */
int sb_tp_split(void* comm, int rank, void** out) {
    *out = NULL;
    if (!have_nccl()) return -5;
    if (!g_nccl.comm_split) {
        sb_set_error("ncclCommSplit not available in this NCCL: two lanes need it");
        return -1;
    }
    ncclComm_t c = NULL;
    int rc = nccl_check(g_nccl.comm_split((ncclComm_t)comm, 0, rank, &c, NULL), "ncclCommSplit");
    *out = rc ? NULL : (void*)c;
    return rc;
}

void sb_tp_destroy(void* comm) {
    if (comm && g_nccl.ok) g_nccl.comm_destroy((ncclComm_t)comm);
}

int sb_tp_allreduce_sum(void* comm, float* buf, size_t n, cudaStream_t st) {
    return nccl_check(g_nccl.all_reduce(buf, buf, n, ncclFloat32, ncclSum, (ncclComm_t)comm, st),
                      "ncclAllReduce");
}

int sb_tp_allgather(void* comm, const void* send, void* recv, size_t bytes, cudaStream_t st) {
    return nccl_check(g_nccl.all_gather(send, recv, bytes, ncclUint8, (ncclComm_t)comm, st),
                      "ncclAllGather");
}
