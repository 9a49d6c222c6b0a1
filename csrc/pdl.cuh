// Programmatic dependent launch helpers (sm_90+ griddepcontrol, used on sm_100a).
//
// A kernel launched with the programmatic stream-serialization attribute may
// start while the previous kernel of its stream is still running;
// grid_dep_wait() blocks (in hardware, no spinning) until that kernel has
// completed and its memory is visible.  Kernels call grid_dep_launch() early so
// that a dependent launch is not held back until their last block exits.  Both
// are no-ops for ordinary launches.
#pragma once

namespace omni {
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" :::); }
}  // namespace omni
