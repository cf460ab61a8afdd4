// Per-call device state of the fused collectives, advanced by a one-thread
// kernel before every call so that a captured CUDA graph replays with fresh
// values.  Host builds of the same functions are tested against the host
// bookkeeping (runtime.Context.next_call) by a protocol model.
#pragma once
#include <cstdint>

namespace tdb {

// GEMM -> reduce-scatter: state {set, expected, epoch, target0, target1}.
// Call `epoch` uses receive set epoch & 1; the counters of that set must reach
// target[set] += signals (cumulative over the calls that used the set).
__host__ __device__ __forceinline__ void advance_rs_state(uint32_t* st, uint32_t signals) {
  const uint32_t e = st[2], s = e & 1u;
  st[3 + s] += signals;
  st[0] = s;
  st[1] = st[3 + s];
  st[2] = e + 1u;
}

// All-gather: state {epoch, parity}; epoch counts calls from 1, the send slot
// alternates with its parity.
__host__ __device__ __forceinline__ void advance_ag_state(uint32_t* st) {
  st[0] += 1u;
  st[1] = st[0] & 1u;
}

}  // namespace tdb
