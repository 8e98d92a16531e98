// The sharded search's communicator object, shared by comm.cpp and the index entry points.
#pragma once

#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "index_impl.h"

typedef struct ncclComm* ncclComm_t;

struct rv_comm {
  int device = 0;
  int rank = 0;
  int world = 1;
  int timeout_ms = 60000;
  ncclComm_t comm = nullptr;
  bool broken = false;  // aborted after a failure or timeout
  std::mutex mu;        // one collective at a time per communicator
  std::string err;
  DevBuf<int64_t> gi;   // gathered [world, count] rows
  DevBuf<double> gs;    // gathered [world, count] f64 scores
};

// All-gathers count (row, f64 score) entries of every rank on stream st and waits (bounded by
// the communicator's time limit) for the result: *gathered_idx / *gathered_score point to
// [world, count] device arrays owned by the communicator.  The caller holds c->mu.
int rv_comm_allgather_lists(rv_comm* c, const int64_t* idx, const double* score, size_t count,
                            int64_t** gathered_idx, double** gathered_score, cudaStream_t st);
