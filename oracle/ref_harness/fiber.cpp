// fiber.cpp — cooperative work-item scheduler for clshim.h (x86-64 System V).
// TEST INFRASTRUCTURE ONLY: it executes the reference's OpenCL C kernels on the
// host so that the oracle restatement can be checked against them.
#include "fiber.h"
#include <cstdlib>
#include <stdexcept>
#include <vector>
#include <omp.h>

// void ojx_fiber_switch(void** save_sp, void* new_sp): saves the callee-saved
// registers on the current stack, stores the stack pointer in *save_sp, loads
// new_sp and restores the registers saved there.
asm(R"(
    .text
    .globl ojx_fiber_switch
    .type ojx_fiber_switch,@function
ojx_fiber_switch:
    pushq %rbp
    pushq %rbx
    pushq %r12
    pushq %r13
    pushq %r14
    pushq %r15
    movq %rsp, (%rdi)
    movq %rsi, %rsp
    popq %r15
    popq %r14
    popq %r13
    popq %r12
    popq %rbx
    popq %rbp
    ret
    .size ojx_fiber_switch, .-ojx_fiber_switch
)");
extern "C" void ojx_fiber_switch(void** save_sp, void* new_sp);

namespace clshim {

thread_local const WorkItem* t_wi = nullptr;

namespace {
constexpr size_t kStack = 64 * 1024;

struct Fiber {
  void* sp = nullptr;
  bool done = false;
  WorkItem wi{};
};

struct Group {
  std::vector<Fiber> fibers;
  std::vector<char> stacks;
  void* sched_sp = nullptr;
  size_t cur = 0;
  const std::function<void()>* call = nullptr;
};

thread_local Group* t_group = nullptr;

[[noreturn]] void fiber_entry() {
  Group* g = t_group;
  Fiber& f = g->fibers[g->cur];
  (*g->call)();
  f.done = true;
  ojx_fiber_switch(&f.sp, g->sched_sp);
  std::abort();  // a finished fiber is never resumed
}

void* init_stack(char* base) {
  uintptr_t top = reinterpret_cast<uintptr_t>(base + kStack) & ~static_cast<uintptr_t>(15);
  void** sp = reinterpret_cast<void**>(top);
  *--sp = nullptr;                                    // fake return address of fiber_entry
  *--sp = reinterpret_cast<void*>(&fiber_entry);      // popped by `ret`
  for (int i = 0; i < 6; ++i) *--sp = nullptr;        // rbp rbx r12 r13 r14 r15
  return sp;
}
}  // namespace

void barrier_yield() {
  Group* g = t_group;
  Fiber& f = g->fibers[g->cur];
  ojx_fiber_switch(&f.sp, g->sched_sp);
}

void run_ndrange(const size_t global[2], const size_t local[2], const std::function<void()>& call) {
  const size_t g3[3] = {global[0], global[1], 1}, l3[3] = {local[0], local[1], 1};
  run_ndrange3(g3, l3, call);
}

void run_ndrange3(const size_t global[3], const size_t local[3], const std::function<void()>& call) {
  if (global[0] % local[0] || global[1] % local[1] || global[2] % local[2])
    throw std::runtime_error("global size must be a multiple of the local size");
  const size_t ng0 = global[0] / local[0], ng1 = global[1] / local[1], ng2 = global[2] / local[2];
  const size_t nwi = local[0] * local[1] * local[2];
  const long long ngroups = static_cast<long long>(ng0 * ng1 * ng2);
#pragma omp parallel
  {
    Group g;
    g.fibers.resize(nwi);
    g.stacks.resize(nwi * kStack);
    g.call = &call;
    t_group = &g;
#pragma omp for schedule(dynamic, 1)
    for (long long gi = 0; gi < ngroups; ++gi) {
      const size_t gx = static_cast<size_t>(gi) % ng0, gy = (static_cast<size_t>(gi) / ng0) % ng1;
      const size_t gz = static_cast<size_t>(gi) / (ng0 * ng1);
      for (size_t i = 0; i < nwi; ++i) {
        Fiber& f = g.fibers[i];
        const size_t lx = i % local[0], ly = (i / local[0]) % local[1], lz = i / (local[0] * local[1]);
        f.done = false;
        f.wi = WorkItem{{gx * local[0] + lx, gy * local[1] + ly, gz * local[2] + lz},
                        {lx, ly, lz},
                        {gx, gy, gz},
                        {local[0], local[1], local[2]},
                        {global[0], global[1], global[2]},
                        {ng0, ng1, ng2}};
        f.sp = init_stack(g.stacks.data() + i * kStack);
      }
      bool alive = true;
      while (alive) {
        alive = false;
        for (size_t i = 0; i < nwi; ++i) {
          Fiber& f = g.fibers[i];
          if (f.done) continue;
          g.cur = i;
          t_wi = &f.wi;
          ojx_fiber_switch(&g.sched_sp, f.sp);
          if (!f.done) alive = true;
        }
      }
    }
    t_group = nullptr;
  }
}

}  // namespace clshim
