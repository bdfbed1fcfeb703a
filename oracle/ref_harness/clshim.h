// clshim.h — lets an OpenCL C kernel file compile as C++ on the host.
//
// TEST INFRASTRUCTURE ONLY (see oracle/README-style header in ojx_oracle.cpp).
// Each work-item runs as a fiber; barrier() hands control back to the
// work-group scheduler in fiber.cpp, which resumes every work-item of the group
// in turn, so a barrier is passed only after every work-item reached it.
// __local variables become per-OS-thread statics: all work-items of one group run
// on the same OS thread, so they share them, as OpenCL requires.
#pragma once
#include <cmath>
#include <cstddef>
#include <cstdint>

namespace clshim {
struct WorkItem {
  size_t gid[3], lid[3], grp[3], lsize[3], gsize[3], ngroups[3];
};
extern thread_local const WorkItem* t_wi;
void barrier_yield();
}  // namespace clshim

#define __kernel
#define kernel
#define __global
#define __constant const
#define __local static thread_local
#define __private
#define CLK_LOCAL_MEM_FENCE 1
#define CLK_GLOBAL_MEM_FENCE 2

typedef _Float16 half;
typedef unsigned int uint;

inline size_t get_global_id(uint d) { return clshim::t_wi->gid[d]; }
inline size_t get_local_id(uint d) { return clshim::t_wi->lid[d]; }
inline size_t get_group_id(uint d) { return clshim::t_wi->grp[d]; }
inline size_t get_local_size(uint d) { return clshim::t_wi->lsize[d]; }
inline size_t get_global_size(uint d) { return clshim::t_wi->gsize[d]; }
inline size_t get_num_groups(uint d) { return clshim::t_wi->ngroups[d]; }
inline void barrier(int) { clshim::barrier_yield(); }

// OpenCL's single-precision builtins for float arguments.
using std::exp;
using std::fabs;
using std::fmax;
using std::fmin;
using std::log;
using std::sqrt;
using std::tanh;
inline float clamp(float x, float lo, float hi) { return fmin(fmax(x, lo), hi); }
