// nccl_comm.cpp -- NCCL communicators and collectives over NVLink / NVSwitch.
//
// Part 1 keeps the reference's API (src/kernels/transformer/tensor_parallel_nccl.cu):
// single-process ncclCommInitAll, group brackets, fp32 in-place all-reduce and
// all-gather.  Unlike the reference's NCCL_CHECK (which only prints), every
// failure is recorded in kc_get_last_error(), and a failed init leaves the
// comms NULL (the reference's own test skips on NULL comms).
// Part 2 adds one-process-per-GPU communicators (unique id + rank) and bf16 /
// fp32 collectives with int status.
#include <nccl.h>

#include <cstring>

#include "kc_common.cuh"

namespace {

int check_nccl(ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return KC_OK;
    return kc::set_error(KC_ERR_NCCL, "%s: %s", what, ncclGetErrorString(r));
}

}  // namespace

extern "C" {

// ----------------------------- reference API ------------------------------
void nccl_comm_init_all(void** comms, int num_comms, const int* devs) {
    if (!comms || num_comms <= 0) {
        kc::set_error(KC_ERR_INVALID_ARG, "nccl_comm_init_all: bad arguments");
        return;
    }
    ncclResult_t r = ncclCommInitAll(reinterpret_cast<ncclComm_t*>(comms), num_comms, devs);
    if (check_nccl(r, "ncclCommInitAll") != KC_OK)
        for (int i = 0; i < num_comms; ++i) comms[i] = nullptr;
}

void nccl_comm_destroy(void* comm) {
    if (comm) check_nccl(ncclCommDestroy(static_cast<ncclComm_t>(comm)), "ncclCommDestroy");
}

void nccl_group_start(void) { check_nccl(ncclGroupStart(), "ncclGroupStart"); }

void nccl_group_end(void) { check_nccl(ncclGroupEnd(), "ncclGroupEnd"); }

void launch_ring_allreduce_nccl(void* comm, float* d_buf, int count, cudaStream_t stream) {
    if (!comm || (!d_buf && count > 0) || count < 0) {
        kc::set_error(KC_ERR_INVALID_ARG, "launch_ring_allreduce_nccl: bad arguments");
        return;
    }
    check_nccl(ncclAllReduce(d_buf, d_buf, (size_t)count, ncclFloat, ncclSum,
                             static_cast<ncclComm_t>(comm), stream),
               "ncclAllReduce");
}

void launch_allgather_nccl(void* comm, const float* d_sendbuf, float* d_recvbuf, int sendcount,
                           cudaStream_t stream) {
    if (!comm || sendcount < 0 || (sendcount > 0 && (!d_sendbuf || !d_recvbuf))) {
        kc::set_error(KC_ERR_INVALID_ARG, "launch_allgather_nccl: bad arguments");
        return;
    }
    check_nccl(ncclAllGather(d_sendbuf, d_recvbuf, (size_t)sendcount, ncclFloat,
                             static_cast<ncclComm_t>(comm), stream),
               "ncclAllGather");
}

int nccl_comm_count(void* comm) {
    int n = 0;
    if (!comm || check_nccl(ncclCommCount(static_cast<ncclComm_t>(comm), &n), "ncclCommCount"))
        return 0;
    return n;
}

int nccl_comm_user_rank(void* comm) {
    int r = -1;
    if (!comm ||
        check_nccl(ncclCommUserRank(static_cast<ncclComm_t>(comm), &r), "ncclCommUserRank"))
        return -1;
    return r;
}

// ------------------------------ kc_* API -----------------------------------
int kc_nccl_unique_id_bytes(void) { return (int)sizeof(ncclUniqueId); }

int kc_nccl_get_unique_id(void* out_id) {
    KC_REQUIRE(out_id, KC_ERR_INVALID_ARG, "null id buffer");
    ncclUniqueId id;
    int st = check_nccl(ncclGetUniqueId(&id), "ncclGetUniqueId");
    if (st) return st;
    std::memcpy(out_id, &id, sizeof(id));
    return KC_OK;
}

int kc_nccl_comm_init_rank(void** comm, int nranks, const void* id, int rank) {
    KC_REQUIRE(comm && id, KC_ERR_INVALID_ARG, "null argument");
    KC_REQUIRE(nranks >= 1 && rank >= 0 && rank < nranks, KC_ERR_INVALID_ARG,
               "rank %d of %d", rank, nranks);
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    ncclComm_t c = nullptr;
    int st = check_nccl(ncclCommInitRank(&c, nranks, uid, rank), "ncclCommInitRank");
    *comm = st ? nullptr : c;
    return st;
}

int kc_nccl_comm_destroy(void* comm) {
    if (!comm) return KC_OK;
    return check_nccl(ncclCommDestroy(static_cast<ncclComm_t>(comm)), "ncclCommDestroy");
}

int kc_nccl_comm_abort(void* comm) {
    if (!comm) return KC_OK;
    return check_nccl(ncclCommAbort(static_cast<ncclComm_t>(comm)), "ncclCommAbort");
}

// Polls a communicator's asynchronous error state: KC_OK, or KC_ERR_NCCL with
// the NCCL message recorded.
int kc_nccl_comm_check(void* comm) {
    KC_REQUIRE(comm, KC_ERR_INVALID_ARG, "null comm");
    ncclResult_t async = ncclSuccess;
    int st = check_nccl(ncclCommGetAsyncError(static_cast<ncclComm_t>(comm), &async),
                        "ncclCommGetAsyncError");
    if (st) return st;
    return check_nccl(async, "async NCCL error");
}

int kc_allgather_bf16(void* comm, const uint16_t* send, uint16_t* recv, long count,
                      cudaStream_t stream) {
    KC_REQUIRE(comm && count >= 0 && (count == 0 || (send && recv)), KC_ERR_INVALID_ARG,
               "kc_allgather_bf16: bad arguments");
    return check_nccl(ncclAllGather(send, recv, (size_t)count, ncclBfloat16,
                                    static_cast<ncclComm_t>(comm), stream),
                      "ncclAllGather(bf16)");
}

int kc_allreduce_bf16(void* comm, const uint16_t* send, uint16_t* recv, long count,
                      cudaStream_t stream) {
    KC_REQUIRE(comm && count >= 0 && (count == 0 || (send && recv)), KC_ERR_INVALID_ARG,
               "kc_allreduce_bf16: bad arguments");
    return check_nccl(ncclAllReduce(send, recv, (size_t)count, ncclBfloat16, ncclSum,
                                    static_cast<ncclComm_t>(comm), stream),
                      "ncclAllReduce(bf16)");
}

int kc_allreduce_f32(void* comm, const float* send, float* recv, long count, cudaStream_t stream) {
    KC_REQUIRE(comm && count >= 0 && (count == 0 || (send && recv)), KC_ERR_INVALID_ARG,
               "kc_allreduce_f32: bad arguments");
    return check_nccl(ncclAllReduce(send, recv, (size_t)count, ncclFloat, ncclSum,
                                    static_cast<ncclComm_t>(comm), stream),
                      "ncclAllReduce(f32)");
}

}  // extern "C"
