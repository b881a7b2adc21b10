// Argument block of the fused ghost-row exchange kernel (halo_exchange.cu), shared with its
// binding. Pointers to peer memory are mapped CUDA IPC allocations.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#define XNN_HALO_MAX_RANKS 8

struct HaloRankArgs {
  const char* src;                          // rows to send from
  const int64_t* rows;                      // source row of each sent row (nullptr: identity)
  int64_t n_send;
  int64_t seg_end[XNN_HALO_MAX_RANKS];      // cumulative sent rows per destination
  int64_t remote_off[XNN_HALO_MAX_RANKS];   // first row in the destination's buffer
  char* out;                                // unpacked rows
  int64_t n_out;
  char* buf[XNN_HALO_MAX_RANKS][2];         // every rank's buffer halves, as mapped here
  unsigned long long* flags[XNN_HALO_MAX_RANKS];  // every rank's counters [world]
  unsigned int* epochs;                     // local, one per CTA
};

struct HaloArgs {
  HaloRankArgs r[XNN_HALO_MAX_RANKS];       // [0] only, unless emulating
  int world;
  int rank;
  int emulate;
  int64_t row_bytes;                        // multiple of 4
  int* status;                              // host-mapped; 0 = ok
  long long timeout_ns;
};

cudaError_t halo_exchange_launch(const HaloArgs& a, int nblocks, cudaStream_t stream);
