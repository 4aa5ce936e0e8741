// Tensor-parallel exchange between the GPUs of one node (one process per GPU).
// The reference runs on a single device and has no counterpart.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <string>

namespace wgd {

struct TpComm;

int tp_handle_size();
int tp_create(TpComm **out, int rank, int size, size_t max_floats, std::string *err);
int tp_export(TpComm *t, void *handle_out, std::string *err);
int tp_open(TpComm *t, const void *handles, std::string *err);
void tp_destroy(TpComm *t);
bool tp_failed(TpComm *t);

// hidden[i] += sum over ranks of partial_r[i] (rank order, identical on every rank).
int tp_allreduce_add(TpComm *t, const float *partial, float *hidden, size_t n, cudaStream_t s, unsigned long long spin_limit,
                     std::string *err);
// buf[i] = sum over ranks of buf_r[i].
int tp_allreduce_inplace(TpComm *t, float *buf, size_t n, cudaStream_t s, unsigned long long spin_limit, std::string *err);
// Each rank holds (idx local to its vocab slice, value); afterwards every rank holds
// the global first maximum (index offset by vocab0 of the owning rank).
int tp_argmax_gather(TpComm *t, int *idx, float *val, int vocab0, cudaStream_t s, unsigned long long spin_limit, std::string *err);
// rows[vocab0 .. vocab0+count) of every rank gathered into rows[0 .. total) on every rank.
int tp_gather_rows(TpComm *t, float *rows, int total, int vocab0, int count, cudaStream_t s, unsigned long long spin_limit,
                   std::string *err);

// The region of the exchange buffers that the persistent decode kernel uses (its own counter,
// candidate tables and partial-row slots, apart from the exchange kernels' slots and flags):
// every rank's buffer base as mapped in this process, and the byte offsets inside a buffer.
struct TpPersistView {
  char *buf[8];
  unsigned long long bar, cand, slot;
};
int tp_persist_view(TpComm *t, TpPersistView *out, std::string *err);

}  // namespace wgd
