// Expert-parallel exchange over NCCL, loaded at run time.
//
// The library does not link NCCL: the first expert-parallel call dlopen()s
// libnccl.so.2 (the copy torch already loaded when torch is in the process),
// so single-GPU users need no NCCL at all. Every call throws swl::Error on
// failure.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

#include <string>

namespace swl {

struct EpComm;

constexpr int EP_ID_BYTES = 128;  // NCCL unique id

// Fills out[EP_ID_BYTES] with a fresh communicator id (one rank makes it and
// hands it to the others out of band).
void ep_unique_id(void* out);
// Joins the communicator of `world` ranks; the calling thread's current CUDA
// device is the rank's device. Blocks until every rank has joined.
EpComm* ep_init(int rank, int world, const void* id);
void ep_destroy(EpComm* c);
// True (with NCCL's message) when the communicator reported an asynchronous
// error, e.g. a peer that went away.
bool ep_async_error(EpComm* c, std::string* why);
// In-place all-gather of `bytes` per rank: buf holds world * bytes, this
// rank's part already at buf + rank * bytes.
void ep_allgather(EpComm* c, void* buf, size_t bytes, cudaStream_t st);
// recv[n] = sum over ranks of send[rank * n + i] (f32).
void ep_reduce_scatter(EpComm* c, const float* send, float* recv, size_t n, cudaStream_t st);
void ep_group_start(EpComm* c);
void ep_group_end(EpComm* c);
// Element-wise int32 maximum over ranks, in place on the device buffer.
void ep_allreduce_i32_max(EpComm* c, int* buf, size_t n, cudaStream_t st);

}  // namespace swl
