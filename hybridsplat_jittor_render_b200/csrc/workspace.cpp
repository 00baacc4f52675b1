// Grow-only device buffers owned by a context (context.h) and the optional
// stage timer.
#include <algorithm>

#include "context.h"

namespace hs {

namespace {
constexpr uint64_t kGranule = 2ull * 1024ull * 1024ull;
}

cudaError_t ensure_buffer(DeviceBuffer& buffer, uint64_t required, uint64_t* growth_count,
                          bool geometric) {
    if (buffer.ptr != nullptr && buffer.bytes >= required) return cudaSuccess;
    // Growth rules of the reference workspaces: the standard backend grows to
    // at least 1.25x the previous capacity (rasterizer/c_api.cpp:85-127), the
    // FlashGS buffers to the requirement (flashgs_backend.cu:56-86); both
    // round up to 2 MiB.
    const uint64_t grown = (!geometric || buffer.bytes == 0)
                               ? required
                               : std::max(required, buffer.bytes + buffer.bytes / 4);
    const uint64_t target = (std::max<uint64_t>(grown, 1) + kGranule - 1) & ~(kGranule - 1);
    void* replacement = nullptr;
    cudaError_t status = cudaMalloc(&replacement, target);
    if (status != cudaSuccess) return status;
    if (buffer.ptr != nullptr) {
        // Work queued earlier may still read the old allocation.
        status = cudaDeviceSynchronize();
        if (status == cudaSuccess) status = cudaFree(buffer.ptr);
        if (status != cudaSuccess) {
            cudaFree(replacement);
            return status;
        }
    }
    buffer.ptr = replacement;
    buffer.bytes = target;
    if (growth_count != nullptr) ++*growth_count;
    return cudaSuccess;
}

cudaError_t release_buffer(DeviceBuffer& buffer) {
    cudaError_t status = cudaSuccess;
    if (buffer.ptr != nullptr) status = cudaFree(buffer.ptr);
    buffer.ptr = nullptr;
    buffer.bytes = 0;
    return status;
}

void StageMarks::start(StageTimer& timer, cudaStream_t stream) {
    stream_ = stream;
    if (!timer.enabled) return;
    if (timer.used >= StageTimer::kMaxPending) {
        ++timer.dropped;
        return;
    }
    if (timer.used == timer.pool.size()) {
        std::array<cudaEvent_t, 4> set{};
        for (auto& e : set) {
            if (cudaEventCreate(&e) != cudaSuccess) {
                ++timer.dropped;
                return;
            }
        }
        timer.pool.push_back(set);
    }
    set_ = &timer.pool[timer.used++];
    mark(0);
}

void StageMarks::mark(int boundary) {
    if (set_ == nullptr) return;
    while (next_ <= boundary && next_ < 4) cudaEventRecord((*set_)[next_++], stream_);
}

StageMarks::~StageMarks() { mark(3); }

cudaError_t stage_timing_read(StageTimer& timer, double out_ms[3], uint64_t* calls) {
    for (size_t i = 0; i < timer.used; ++i) {
        auto& set = timer.pool[i];
        cudaError_t st = cudaEventSynchronize(set[3]);
        if (st != cudaSuccess) return st;
        for (int k = 0; k < 3; ++k) {
            float ms = 0.0f;
            st = cudaEventElapsedTime(&ms, set[k], set[k + 1]);
            if (st != cudaSuccess) return st;
            timer.total_ms[k] += ms;
        }
        ++timer.calls;
    }
    timer.used = 0;
    for (int k = 0; k < 3; ++k) out_ms[k] = timer.total_ms[k];
    if (calls != nullptr) *calls = timer.calls;
    timer.total_ms[0] = timer.total_ms[1] = timer.total_ms[2] = 0.0;
    timer.calls = 0;
    return cudaSuccess;
}

cudaError_t ensure_device_error(HsRasterizerContext* context) {
    if (context->device_error != nullptr) return cudaSuccess;
    void* p = nullptr;
    cudaError_t st = cudaMalloc(&p, 256);
    if (st != cudaSuccess) return st;
    st = cudaMemset(p, 0, 256);
    if (st != cudaSuccess) {
        cudaFree(p);
        return st;
    }
    context->device_error = static_cast<uint32_t*>(p);
    return cudaSuccess;
}

cudaError_t ensure_side_stream(HsRasterizerContext* context) {
    cudaError_t st = cudaSuccess;
    if (context->side_stream == nullptr)
        st = cudaStreamCreateWithFlags(&context->side_stream, cudaStreamNonBlocking);
    if (st == cudaSuccess && context->side_event == nullptr)
        st = cudaEventCreateWithFlags(&context->side_event, cudaEventDisableTiming);
    if (st == cudaSuccess && context->fork_event == nullptr)
        st = cudaEventCreateWithFlags(&context->fork_event, cudaEventDisableTiming);
    return st;
}

cudaError_t ensure_post_stream(HsRasterizerContext* context) {
    cudaError_t st = cudaSuccess;
    if (context->post_stream == nullptr)
        st = cudaStreamCreateWithFlags(&context->post_stream, cudaStreamNonBlocking);
    if (st == cudaSuccess && context->post_fork_event == nullptr)
        st = cudaEventCreateWithFlags(&context->post_fork_event, cudaEventDisableTiming);
    if (st == cudaSuccess && context->post_done_event == nullptr)
        st = cudaEventCreateWithFlags(&context->post_done_event, cudaEventDisableTiming);
    return st;
}

cudaError_t ensure_graph_streams(HsRasterizerContext* context) {
    cudaError_t st = cudaSuccess;
    if (context->signal_stream == nullptr)
        st = cudaStreamCreateWithFlags(&context->signal_stream, cudaStreamNonBlocking);
    for (cudaEvent_t* e : {&context->signal_event, &context->graph_fork_event, &context->graph_join_event}) {
        if (st == cudaSuccess && *e == nullptr) st = cudaEventCreateWithFlags(e, cudaEventDisableTiming);
    }
    return st;
}

void destroy_view_graphs(HsRasterizerContext* context) {
    // an executable still in flight is freed when it completes
    for (HsRasterizerContext::ViewGraph& g : context->view_graphs) {
        if (g.exec != nullptr) cudaGraphExecDestroy(g.exec);
    }
    context->view_graphs.clear();
    context->view_recent_keys.clear();
}

void destroy_side_stream(HsRasterizerContext* context) {
    destroy_view_graphs(context);
    if (context->signal_stream != nullptr) cudaStreamDestroy(context->signal_stream);
    for (cudaEvent_t* e : {&context->signal_event, &context->graph_fork_event, &context->graph_join_event}) {
        if (*e != nullptr) cudaEventDestroy(*e);
        *e = nullptr;
    }
    context->signal_stream = nullptr;
    if (context->side_stream != nullptr) cudaStreamDestroy(context->side_stream);
    if (context->side_event != nullptr) cudaEventDestroy(context->side_event);
    if (context->fork_event != nullptr) cudaEventDestroy(context->fork_event);
    if (context->post_stream != nullptr) cudaStreamDestroy(context->post_stream);
    if (context->post_fork_event != nullptr) cudaEventDestroy(context->post_fork_event);
    if (context->post_done_event != nullptr) cudaEventDestroy(context->post_done_event);
    context->side_stream = nullptr;
    context->side_event = nullptr;
    context->fork_event = nullptr;
    context->post_stream = nullptr;
    context->post_fork_event = nullptr;
    context->post_done_event = nullptr;
}

void stage_timing_destroy(StageTimer& timer) {
    for (auto& set : timer.pool)
        for (auto& e : set) cudaEventDestroy(e);
    timer.pool.clear();
    timer.used = 0;
}

}  // namespace hs
