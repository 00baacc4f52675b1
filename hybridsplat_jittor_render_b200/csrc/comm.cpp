// NCCL communicator of the multi-GPU replicas (one process per GPU).
//
// The forward renderer shards with no per-frame exchange: every GPU holds a
// full replica of the Gaussians and renders its own views or its own strip of
// tile rows. The only collectives are at session start (one broadcast of the
// scene arrays from the root rank straight into each rank's device buffers)
// and a few host values (per-rank timings, a barrier). This file provides
// them behind the C ABI so that a host without a deep-learning framework can
// run the multi-GPU session; the reference has no multi-GPU path.
//
// libnccl.so.2 is loaded on first use with dlopen (a process that already
// holds an NCCL, for example through a framework, reuses that copy). Every
// communicator is created non-blocking and every operation is polled against
// a deadline: a rank that never joins, or dies mid-operation, turns into an
// HS_STATUS_CUDA_ERROR on the others (the communicator is then aborted)
// instead of a hang.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>

#include <cuda_runtime.h>

#include "hybridsplat_b200_ext.h"

struct HsB200Comm {
    int32_t device = 0;
    int32_t rank = 0;
    int32_t rank_count = 0;
    double timeout_s = 120.0;
    ncclComm_t comm = nullptr;
    cudaStream_t stream = nullptr;
    double* scratch = nullptr;  // device buffer of kScratchValues doubles
};

namespace {

constexpr uint32_t kScratchValues = 512;

struct NcclApi {
    bool loaded = false;
    std::string error;
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*abort)(ncclComm_t) = nullptr;
    ncclResult_t (*destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*finalize)(ncclComm_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
};

NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (lib == nullptr) lib = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (lib == nullptr) {
            const char* why = dlerror();
            api.error = std::string("cannot load libnccl.so.2: ") + (why ? why : "unknown");
            return;
        }
        auto sym = [&](const char* name) -> void* { return dlsym(lib, name); };
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
        api.init_rank_config =
            reinterpret_cast<decltype(api.init_rank_config)>(sym("ncclCommInitRankConfig"));
        api.broadcast = reinterpret_cast<decltype(api.broadcast)>(sym("ncclBroadcast"));
        api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(sym("ncclAllReduce"));
        api.get_async_error =
            reinterpret_cast<decltype(api.get_async_error)>(sym("ncclCommGetAsyncError"));
        api.abort = reinterpret_cast<decltype(api.abort)>(sym("ncclCommAbort"));
        api.destroy = reinterpret_cast<decltype(api.destroy)>(sym("ncclCommDestroy"));
        api.finalize = reinterpret_cast<decltype(api.finalize)>(sym("ncclCommFinalize"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
        if (!api.get_unique_id || !api.init_rank_config || !api.broadcast || !api.all_reduce ||
            !api.get_async_error || !api.abort || !api.destroy || !api.error_string) {
            api.error = "libnccl.so.2 lacks a required entry point";
            return;
        }
        api.loaded = true;
    });
    return api;
}

void write_text(char* destination, uint64_t capacity, const std::string& text) noexcept {
    if (destination == nullptr || capacity == 0) return;
    const size_t n = std::min<size_t>(text.size(), capacity - 1);
    if (n != 0) std::memcpy(destination, text.data(), n);
    destination[n] = '\0';
}

int32_t fail(HsStatus status, const std::string& text, char* error_text, uint64_t capacity) {
    write_text(error_text, capacity, text);
    return static_cast<int32_t>(status);
}

int32_t ok(char* error_text, uint64_t capacity) {
    write_text(error_text, capacity, "");
    return HS_STATUS_OK;
}

std::string nccl_text(const char* what, ncclResult_t r) {
    NcclApi& api = nccl();
    return std::string(what) + ": " + (api.error_string ? api.error_string(r) : "NCCL error");
}

// Restores the caller's current device on scope exit.
class DeviceScope {
public:
    explicit DeviceScope(int device) {
        had_ = cudaGetDevice(&previous_) == cudaSuccess;
        status_ = cudaSetDevice(device);
    }
    ~DeviceScope() {
        if (had_) cudaSetDevice(previous_);
    }
    cudaError_t status() const { return status_; }

private:
    int previous_ = 0;
    bool had_ = false;
    cudaError_t status_ = cudaSuccess;
};

using Clock = std::chrono::steady_clock;

// Polls the communicator (and, when given, the stream) until the pending
// operation completes, fails or the deadline passes; on failure or timeout
// the communicator is aborted and becomes unusable.
int32_t settle(HsB200Comm* c, cudaStream_t stream, const char* what, char* error_text,
               uint64_t capacity) {
    NcclApi& api = nccl();
    const auto deadline = Clock::now() + std::chrono::duration<double>(c->timeout_s);
    for (;;) {
        ncclResult_t state = ncclSuccess;
        const ncclResult_t q = api.get_async_error(c->comm, &state);
        if (q != ncclSuccess) state = q;
        if (state != ncclSuccess && state != ncclInProgress) {
            api.abort(c->comm);
            c->comm = nullptr;
            return fail(HS_STATUS_CUDA_ERROR, nccl_text(what, state), error_text, capacity);
        }
        if (state == ncclSuccess) {
            const cudaError_t s = stream != nullptr ? cudaStreamQuery(stream) : cudaSuccess;
            if (s == cudaSuccess) return HS_STATUS_OK;
            if (s != cudaErrorNotReady) {
                return fail(HS_STATUS_CUDA_ERROR, std::string(what) + ": " + cudaGetErrorString(s),
                            error_text, capacity);
            }
        }
        if (Clock::now() > deadline) {
            api.abort(c->comm);
            c->comm = nullptr;
            char text[160];
            std::snprintf(text, sizeof(text),
                          "%s: not complete after %.1f s (a rank did not join or left); communicator aborted",
                          what, c->timeout_s);
            return fail(HS_STATUS_CUDA_ERROR, text, error_text, capacity);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

int32_t check_comm(HsB200Comm* c, char* error_text, uint64_t capacity) {
    if (c == nullptr) return fail(HS_STATUS_INVALID_ARGUMENT, "communicator is null", error_text, capacity);
    if (c->comm == nullptr) {
        return fail(HS_STATUS_INVALID_ARGUMENT, "communicator was aborted after an earlier failure",
                    error_text, capacity);
    }
    return HS_STATUS_OK;
}

// One reduction of host doubles through the device scratch buffer.
int32_t reduce_host(HsB200Comm* c, const double* in, double* out, uint32_t count, ncclRedOp_t op,
                    const char* what, char* error_text, uint64_t capacity) {
    NcclApi& api = nccl();
    DeviceScope scope(c->device);
    if (scope.status() != cudaSuccess)
        return fail(HS_STATUS_CUDA_ERROR, cudaGetErrorString(scope.status()), error_text, capacity);
    cudaError_t e = cudaMemcpyAsync(c->scratch, in, count * sizeof(double), cudaMemcpyHostToDevice,
                                    c->stream);
    if (e != cudaSuccess) return fail(HS_STATUS_CUDA_ERROR, cudaGetErrorString(e), error_text, capacity);
    const ncclResult_t r = api.all_reduce(c->scratch, c->scratch, count, ncclFloat64, op, c->comm, c->stream);
    if (r != ncclSuccess && r != ncclInProgress) {
        return fail(HS_STATUS_CUDA_ERROR, nccl_text(what, r), error_text, capacity);
    }
    const int32_t s = settle(c, c->stream, what, error_text, capacity);
    if (s != HS_STATUS_OK) return s;
    e = cudaMemcpyAsync(out, c->scratch, count * sizeof(double), cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) return fail(HS_STATUS_CUDA_ERROR, cudaGetErrorString(e), error_text, capacity);
    return HS_STATUS_OK;
}

}  // namespace

extern "C" {

int32_t hs_b200_comm_unique_id_v1(uint8_t* id128, char* error_text, uint64_t error_capacity) noexcept {
    if (error_capacity != 0 && error_text == nullptr) return HS_STATUS_INVALID_ARGUMENT;
    if (id128 == nullptr) return fail(HS_STATUS_INVALID_ARGUMENT, "id128 is null", error_text, error_capacity);
    NcclApi& api = nccl();
    if (!api.loaded) return fail(HS_STATUS_INTERNAL_ERROR, api.error, error_text, error_capacity);
    static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id size");
    ncclUniqueId id;
    const ncclResult_t r = api.get_unique_id(&id);
    if (r != ncclSuccess) return fail(HS_STATUS_CUDA_ERROR, nccl_text("ncclGetUniqueId", r), error_text, error_capacity);
    std::memcpy(id128, &id, sizeof(id));
    return ok(error_text, error_capacity);
}

int32_t hs_b200_comm_create_v1(int32_t device, int32_t rank_count, int32_t rank, const uint8_t* id128,
                               double timeout_s, HsB200CommHandle* out_comm, char* error_text,
                               uint64_t error_capacity) noexcept {
    if (error_capacity != 0 && error_text == nullptr) return HS_STATUS_INVALID_ARGUMENT;
    if (id128 == nullptr || out_comm == nullptr) {
        return fail(HS_STATUS_INVALID_ARGUMENT, "id128 or out_comm is null", error_text, error_capacity);
    }
    *out_comm = nullptr;
    if (rank_count <= 0 || rank < 0 || rank >= rank_count || !std::isfinite(timeout_s) || timeout_s <= 0.0) {
        return fail(HS_STATUS_RANGE_ERROR, "rank, rank_count or timeout is out of range", error_text,
                    error_capacity);
    }
    NcclApi& api = nccl();
    if (!api.loaded) return fail(HS_STATUS_INTERNAL_ERROR, api.error, error_text, error_capacity);
    try {
        DeviceScope scope(device);
        if (scope.status() != cudaSuccess) {
            return fail(HS_STATUS_CUDA_ERROR, std::string("cudaSetDevice: ") + cudaGetErrorString(scope.status()),
                        error_text, error_capacity);
        }
        HsB200Comm* c = new HsB200Comm();
        c->device = device;
        c->rank = rank;
        c->rank_count = rank_count;
        c->timeout_s = timeout_s;
        cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaMalloc(&c->scratch, kScratchValues * sizeof(double));
        if (e != cudaSuccess) {
            if (c->stream) cudaStreamDestroy(c->stream);
            delete c;
            return fail(e == cudaErrorMemoryAllocation ? HS_STATUS_OUT_OF_MEMORY : HS_STATUS_CUDA_ERROR,
                        cudaGetErrorString(e), error_text, error_capacity);
        }
        ncclUniqueId id;
        std::memcpy(&id, id128, sizeof(id));
        ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
        config.blocking = 0;
        const ncclResult_t r = api.init_rank_config(&c->comm, rank_count, id, rank, &config);
        int32_t s = HS_STATUS_OK;
        if (r != ncclSuccess && r != ncclInProgress) {
            s = fail(HS_STATUS_CUDA_ERROR, nccl_text("ncclCommInitRankConfig", r), error_text, error_capacity);
            if (c->comm) api.abort(c->comm);
            c->comm = nullptr;
        } else {
            s = settle(c, nullptr, "NCCL communicator initialisation", error_text, error_capacity);
        }
        if (s != HS_STATUS_OK) {
            cudaFree(c->scratch);
            cudaStreamDestroy(c->stream);
            delete c;
            return s;
        }
        *out_comm = c;
        return ok(error_text, error_capacity);
    } catch (const std::exception& ex) {
        return fail(HS_STATUS_INTERNAL_ERROR, ex.what(), error_text, error_capacity);
    }
}

int32_t hs_b200_comm_broadcast_v1(HsB200CommHandle comm, void* buffer, uint64_t bytes, int32_t root,
                                  void* stream, char* error_text, uint64_t error_capacity) noexcept {
    if (error_capacity != 0 && error_text == nullptr) return HS_STATUS_INVALID_ARGUMENT;
    const int32_t cs = check_comm(comm, error_text, error_capacity);
    if (cs != HS_STATUS_OK) return cs;
    if (root < 0 || root >= comm->rank_count) {
        return fail(HS_STATUS_RANGE_ERROR, "root is not a rank of the communicator", error_text, error_capacity);
    }
    if (bytes == 0) return ok(error_text, error_capacity);
    if (buffer == nullptr) return fail(HS_STATUS_INVALID_ARGUMENT, "buffer is null", error_text, error_capacity);
    DeviceScope scope(comm->device);
    if (scope.status() != cudaSuccess)
        return fail(HS_STATUS_CUDA_ERROR, cudaGetErrorString(scope.status()), error_text, error_capacity);
    // Work queued on the caller's stream (that filled the root's buffer) comes
    // first; the caller's stream then waits for the broadcast.
    cudaStream_t user = static_cast<cudaStream_t>(stream);
    cudaEvent_t ev = nullptr;
    cudaError_t e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventRecord(ev, user);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(comm->stream, ev, 0);
    if (e != cudaSuccess) {
        if (ev) cudaEventDestroy(ev);
        return fail(HS_STATUS_CUDA_ERROR, cudaGetErrorString(e), error_text, error_capacity);
    }
    NcclApi& api = nccl();
    const ncclResult_t r = api.broadcast(buffer, buffer, bytes, ncclChar, root, comm->comm, comm->stream);
    int32_t s = HS_STATUS_OK;
    if (r != ncclSuccess && r != ncclInProgress) {
        s = fail(HS_STATUS_CUDA_ERROR, nccl_text("ncclBroadcast", r), error_text, error_capacity);
    } else {
        s = settle(comm, comm->stream, "scene broadcast", error_text, error_capacity);
    }
    if (s == HS_STATUS_OK) {
        e = cudaEventRecord(ev, comm->stream);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(user, ev, 0);
        if (e != cudaSuccess) s = fail(HS_STATUS_CUDA_ERROR, cudaGetErrorString(e), error_text, error_capacity);
    }
    cudaEventDestroy(ev);
    return s == HS_STATUS_OK ? ok(error_text, error_capacity) : s;
}

int32_t hs_b200_comm_allreduce_max_f64_v1(HsB200CommHandle comm, const double* values, double* out,
                                          uint32_t count, char* error_text, uint64_t error_capacity) noexcept {
    if (error_capacity != 0 && error_text == nullptr) return HS_STATUS_INVALID_ARGUMENT;
    const int32_t cs = check_comm(comm, error_text, error_capacity);
    if (cs != HS_STATUS_OK) return cs;
    if (count == 0) return ok(error_text, error_capacity);
    if (values == nullptr || out == nullptr) {
        return fail(HS_STATUS_INVALID_ARGUMENT, "values or out is null", error_text, error_capacity);
    }
    if (count > kScratchValues) {
        return fail(HS_STATUS_RANGE_ERROR, "at most 512 values per reduction", error_text, error_capacity);
    }
    const int32_t s = reduce_host(comm, values, out, count, ncclMax, "host-value max reduction", error_text,
                                  error_capacity);
    return s == HS_STATUS_OK ? ok(error_text, error_capacity) : s;
}

int32_t hs_b200_comm_barrier_v1(HsB200CommHandle comm, char* error_text, uint64_t error_capacity) noexcept {
    if (error_capacity != 0 && error_text == nullptr) return HS_STATUS_INVALID_ARGUMENT;
    const int32_t cs = check_comm(comm, error_text, error_capacity);
    if (cs != HS_STATUS_OK) return cs;
    const double one = 1.0;
    double sum = 0.0;
    const int32_t s = reduce_host(comm, &one, &sum, 1, ncclSum, "barrier", error_text, error_capacity);
    return s == HS_STATUS_OK ? ok(error_text, error_capacity) : s;
}

int32_t hs_b200_comm_destroy_v1(HsB200CommHandle comm, char* error_text, uint64_t error_capacity) noexcept {
    if (error_capacity != 0 && error_text == nullptr) return HS_STATUS_INVALID_ARGUMENT;
    if (comm == nullptr) return ok(error_text, error_capacity);
    NcclApi& api = nccl();
    int32_t s = HS_STATUS_OK;
    {
        DeviceScope scope(comm->device);
        if (comm->comm != nullptr) {
            if (api.finalize != nullptr) {
                const ncclResult_t r = api.finalize(comm->comm);
                if (r == ncclSuccess || r == ncclInProgress) {
                    s = settle(comm, nullptr, "communicator finalize", error_text, error_capacity);
                }
            }
            if (comm->comm != nullptr) api.destroy(comm->comm);
        }
        if (comm->scratch) cudaFree(comm->scratch);
        if (comm->stream) cudaStreamDestroy(comm->stream);
    }
    delete comm;
    return s == HS_STATUS_OK ? ok(error_text, error_capacity) : s;
}

}  // extern "C"
