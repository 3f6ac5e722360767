// runtime.h - the multi-GPU runtime behind cdclq_runtime* (runtime.cu), shared with the model pipeline (model.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

#include "cdclq.h"

namespace cdclq {

// One rank of the runtime: its device, its stream, and (nranks > 1) the NCCL communicator.
struct Runtime {
    int device = 0;
    int nranks = 1;
    int rank = 0;
    double timeout_s = 600.0;
    cudaStream_t st = nullptr;
    cudaStream_t comm_st = nullptr;  // collectives that overlap work on st (the factor broadcasts)
    void* comm = nullptr;      // ncclComm_t
    bool broken = false;       // a collective failed or timed out: the communicator was aborted
    int32_t* flag_dev = nullptr;  // 2 ints: error consensus
    char* msg_dev = nullptr;      // 512 bytes: the failing rank's message
    bool owned_stream = false;
};

// Contiguous row range [r0, r1) of `rank` in whole row chunks of `row_chunk` rows; `rotate` (the layer index)
// shifts which rank takes which range so that leftover chunks of consecutive layers land on different ranks.
void shard_rows(size_t d_out, size_t row_chunk, int rank, int nranks, size_t rotate, size_t* r0, size_t* r1);
// The rank whose range is the first one (rows from 0) of a layer with `rotate`.
int first_range_rank(int nranks, size_t rotate);
// Owners by longest-processing-time on n^power, largest first, ties by index, to the least-loaded rank.
std::vector<int> assign_owners(const std::vector<size_t>& ns, int nranks, int power);

// Collectives on rt->st (no-ops with one rank).  Grouped calls between group_begin / group_end run together.
int rt_group_begin(Runtime* rt);
int rt_group_end(Runtime* rt);
int rt_broadcast(Runtime* rt, void* buf, size_t bytes, int root);
int rt_broadcast_on(Runtime* rt, cudaStream_t stream, void* buf, size_t bytes, int root);
int rt_send(Runtime* rt, const void* buf, size_t bytes, int peer);
int rt_recv(Runtime* rt, void* buf, size_t bytes, int peer);
int rt_allreduce_sum_f64(Runtime* rt, double* buf_dev, size_t count);
int rt_allreduce_sum_u64(Runtime* rt, uint64_t* buf_dev, size_t count);
int rt_allreduce_max_u64(Runtime* rt, uint64_t* buf_dev, size_t count);
// Waits for rt->st with the runtime's timeout; on a timeout or an NCCL failure the communicator is aborted.
int rt_sync(Runtime* rt);
// Every rank passes its local status; all return the first failing rank's status, the ranks that did not fail
// with "rank <r> failed: <its message>".  Collective: every rank calls it at the same points.
int rt_agree(Runtime* rt, int rc);

// Quantize a batch over the runtime's ranks: rows of every layer sharded in whole row chunks, factors computed
// by their owner ranks and broadcast, statistics all-reduced, outputs optionally gathered on rank 0.  Layer
// descriptors describe FULL layers (w and the outputs point at row 0).
int runtime_quantize_batch(Runtime* rt, const cdclq_batch_input* inputs, size_t n_inputs,
                           const cdclq_batch_layer* layers, size_t n_layers, const cdclq_config& cfg, bool on_device,
                           bool gather);

// engine.cu
int ensure_device();
int layer_perm(const float* h_dev, size_t n, const double* colsq, const cdclq_config& cfg, std::vector<uint32_t>& perm,
               std::vector<uint8_t>& gbits, size_t& nskel, cudaStream_t st);

}  // namespace cdclq
