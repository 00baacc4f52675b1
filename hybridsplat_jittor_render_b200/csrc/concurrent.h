// Concurrent execution of independent raster calls.
//
// A raster call reads back its pair totals between preprocess and binning and
// its wait-status word after binning, so a call is split into four phases
// that wait on nothing but those two readbacks:
//   begin()   workspaces, preprocess, totals readback, depth sort;
//   bin()     waits for the totals, queues emission, tile sort, ranges;
//   render()  queues the tile renderer;
//   finish()  waits for the end of binning and fails the call if one of its
//             bounded waits gave up (the renderer is already queued).
// run_many() puts every call on its context's side stream and queues all
// begin() phases, then all bin() phases, then all render() phases, then
// runs all finish() phases. The renderers are persistent grids that fill the
// GPU, so each waits for the binning of every call: the latency-bound
// preprocess and sorting stages of the calls overlap one another instead of
// queueing behind a renderer.
#pragma once

#include <memory>
#include <vector>

#include "context.h"

namespace hs {

// raster_begin (optional) is recorded when every call's binning is done and
// the renderers may start, for callers that time other traffic around them.
// finish false leaves out the finish() phases (calls captured into a graph,
// whose status the capturer reads after each replay).
template <class Pass, class Call>
cudaError_t run_many(HsRasterizerContext* const* contexts, const Call* calls, uint32_t count,
                     cudaStream_t stream, cudaEvent_t raster_begin = nullptr, bool finish = true) {
    if (count == 0) return cudaSuccess;
    for (uint32_t i = 0; i < count; ++i) {
        const cudaError_t st = ensure_side_stream(contexts[i]);
        if (st != cudaSuccess) return st;
    }
    cudaError_t st = cudaEventRecord(contexts[0]->fork_event, stream);
    if (st != cudaSuccess) return st;
    for (uint32_t i = 0; i < count; ++i) {
        st = cudaStreamWaitEvent(contexts[i]->side_stream, contexts[0]->fork_event, 0);
        if (st != cudaSuccess) return st;
    }
    std::vector<std::unique_ptr<Pass>> passes;
    passes.reserve(count);
    for (uint32_t i = 0; i < count; ++i) {
        Call call = calls[i];
        call.stream = contexts[i]->side_stream;
        passes.emplace_back(new Pass(contexts[i], call));
    }
    for (auto& p : passes)
        if (st == cudaSuccess) st = p->begin();
    for (auto& p : passes)
        if (st == cudaSuccess) st = p->bin();
    if (st == cudaSuccess && count > 1) {
        for (uint32_t i = 0; i < count && st == cudaSuccess; ++i)
            st = cudaEventRecord(contexts[i]->side_event, contexts[i]->side_stream);
        for (uint32_t i = 0; i < count && st == cudaSuccess; ++i) {
            for (uint32_t j = 0; j < count && st == cudaSuccess; ++j) {
                if (j != i) st = cudaStreamWaitEvent(contexts[i]->side_stream, contexts[j]->side_event, 0);
            }
        }
    }
    // contexts[0]'s side stream has waited for every call's binning
    if (st == cudaSuccess && raster_begin != nullptr)
        st = cudaEventRecord(raster_begin, contexts[0]->side_stream);
    for (auto& p : passes)
        if (st == cudaSuccess) st = p->render();
    for (auto& p : passes)
        if (st == cudaSuccess && finish) st = p->finish();
    // Join also after an error: the caller's stream stays ordered after
    // everything that was queued.
    for (uint32_t i = 0; i < count; ++i) {
        const cudaError_t r = cudaEventRecord(contexts[i]->side_event, contexts[i]->side_stream);
        const cudaError_t w = r == cudaSuccess ? cudaStreamWaitEvent(stream, contexts[i]->side_event, 0) : r;
        if (st == cudaSuccess) st = w;
    }
    return st;
}

}  // namespace hs
