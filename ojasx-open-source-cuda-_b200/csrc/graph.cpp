// graph.cpp — CUDA Graph capture and replay of ojx launches.
//
// The reference records pyopencl kernel calls into a Python list and replays
// them one host call at a time (torchcl/jit/graph_runner.py:35-90).  Here a
// stream capture records the launches and one cudaGraphLaunch submits the whole
// sequence, so a replay costs one host call however many kernels it holds.
//
// Scratch: a launch that needs a workspace while its stream is being captured
// gets a fresh buffer owned by the capture (capture_workspace below) instead of
// the stream's shared workspace, which a later ordinary launch could grow (free
// and reallocate) under the graph.  Buffers that must start at zero (the skinny
// route's arrival counters) are cleared once, on a private stream, when they
// are allocated; the kernels return those counters to zero themselves, so every
// replay finds them cleared.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/ojx.h"
#include "internal.h"

struct ojx_graph_s {
  int device = 0;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  std::vector<void*> owned;             // workspaces of the captured launches
  std::vector<cudaGraphNode_t> order;   // nodes in execution (topological) order
  int32_t kernel_nodes = 0;
};

namespace ojx {
namespace {

struct Capture {
  int device = 0;
  std::vector<void*> owned;
};

std::mutex g_cap_mu;
std::map<cudaStream_t, Capture>& captures() {
  static auto* m = new std::map<cudaStream_t, Capture>();
  return *m;
}

// Private stream (per device) used to clear capture-owned buffers while the
// captured stream is recording.
cudaStream_t clear_stream(int dev) {
  static std::mutex mu;
  static std::map<int, cudaStream_t>* m = new std::map<int, cudaStream_t>();
  std::lock_guard<std::mutex> g(mu);
  auto it = m->find(dev);
  if (it != m->end()) return it->second;
  cudaStream_t s = nullptr;
  if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) return nullptr;
  (*m)[dev] = s;
  return s;
}

void free_all(std::vector<void*>& v) {
  for (void* p : v) cudaFree(p);
  v.clear();
}

// Topological order of the graph (Kahn), ties broken by cudaGraphGetNodes order.
int order_nodes(cudaGraph_t graph, std::vector<cudaGraphNode_t>& out) {
  size_t n = 0;
  if (int st = cuda_status(cudaGraphGetNodes(graph, nullptr, &n), "cudaGraphGetNodes")) return st;
  std::vector<cudaGraphNode_t> nodes(n);
  if (n && (cuda_status(cudaGraphGetNodes(graph, nodes.data(), &n), "cudaGraphGetNodes")))
    return OJX_ERR_CUDA;
  size_t ne = 0;
  if (int st = cuda_status(cudaGraphGetEdges(graph, nullptr, nullptr, &ne), "cudaGraphGetEdges"))
    return st;
  std::vector<cudaGraphNode_t> from(ne), to(ne);
  if (ne && cuda_status(cudaGraphGetEdges(graph, from.data(), to.data(), &ne), "cudaGraphGetEdges"))
    return OJX_ERR_CUDA;
  std::map<cudaGraphNode_t, size_t> idx;
  for (size_t i = 0; i < n; ++i) idx[nodes[i]] = i;
  std::vector<int> indeg(n, 0);
  std::vector<std::vector<size_t>> succ(n);
  for (size_t e = 0; e < ne; ++e) {
    const size_t a = idx[from[e]], b = idx[to[e]];
    succ[a].push_back(b);
    ++indeg[b];
  }
  std::vector<size_t> ready;
  for (size_t i = 0; i < n; ++i)
    if (!indeg[i]) ready.push_back(i);
  out.clear();
  while (!ready.empty()) {
    auto it = std::min_element(ready.begin(), ready.end());
    const size_t i = *it;
    ready.erase(it);
    out.push_back(nodes[i]);
    for (size_t j : succ[i])
      if (--indeg[j] == 0) ready.push_back(j);
  }
  return out.size() == n ? OJX_OK : set_error(OJX_ERR_CUDA, "captured graph has a cycle");
}

// "_ZN3ojx14tc_gemm_kernelILi0E..." -> "ojx::tc_gemm_kernel"; plain names unchanged.
void short_name(const char* mangled, char* out, size_t cap) {
  out[0] = 0;
  if (!mangled) return;
  const char* p = mangled;
  if (std::strncmp(p, "_Z", 2) != 0) {
    std::snprintf(out, cap, "%s", mangled);
    return;
  }
  p += 2;
  if (*p == 'N') ++p;
  std::string r;
  while (*p >= '0' && *p <= '9') {
    size_t len = 0;
    while (*p >= '0' && *p <= '9') len = len * 10 + static_cast<size_t>(*p++ - '0');
    if (std::strlen(p) < len) break;
    if (!r.empty()) r += "::";
    r.append(p, len);
    p += len;
  }
  std::snprintf(out, cap, "%s", r.empty() ? mangled : r.c_str());
}

}  // namespace

void* capture_workspace(cudaStream_t s, size_t bytes, bool zero) {
  std::lock_guard<std::mutex> g(g_cap_mu);
  auto it = captures().find(s);
  if (it == captures().end()) {
    set_error(OJX_ERR_UNSUPPORTED,
              "the stream is being captured outside ojx_graph_capture_begin; a launch that needs "
              "scratch memory cannot be recorded there");
    return nullptr;
  }
  const size_t nb = (std::max<size_t>(bytes, 1) + 255) / 256 * 256;
  void* p = nullptr;
  if (cuda_status(cudaMalloc(&p, nb), "capture workspace cudaMalloc")) return nullptr;
  if (zero) {
    cudaStream_t cs = clear_stream(it->second.device);
    if (!cs || cuda_status(cudaMemsetAsync(p, 0, nb, cs), "capture workspace clear") ||
        cuda_status(cudaStreamSynchronize(cs), "capture workspace clear")) {
      cudaFree(p);
      return nullptr;
    }
  }
  it->second.owned.push_back(p);
  return p;
}

}  // namespace ojx

using namespace ojx;

extern "C" {

int ojx_graph_capture_begin(ojx_stream s) {
  cudaStream_t cs = static_cast<cudaStream_t>(s);
  if (!cs) return set_error(OJX_ERR_INVALID, "graph capture needs a stream from ojx_stream_create");
  int dev = 0;
  if (int st = cuda_status(cudaGetDevice(&dev), "cudaGetDevice")) return st;
  {
    std::lock_guard<std::mutex> g(g_cap_mu);
    if (captures().count(cs)) return set_error(OJX_ERR_INVALID, "the stream is already capturing");
    captures()[cs] = Capture{dev, {}};
  }
  int st = cuda_status(cudaStreamBeginCapture(cs, cudaStreamCaptureModeRelaxed),
                       "cudaStreamBeginCapture");
  if (st) {
    std::lock_guard<std::mutex> g(g_cap_mu);
    captures().erase(cs);
  }
  return st;
}

int ojx_graph_capture_end(ojx_stream s, ojx_graph* out) {
  cudaStream_t cs = static_cast<cudaStream_t>(s);
  if (!out) return set_error(OJX_ERR_INVALID, "out is NULL");
  *out = nullptr;
  Capture cap;
  {
    std::lock_guard<std::mutex> g(g_cap_mu);
    auto it = captures().find(cs);
    if (it == captures().end())
      return set_error(OJX_ERR_INVALID, "the stream is not capturing (ojx_graph_capture_begin)");
    cap = std::move(it->second);
    captures().erase(it);
  }
  cudaGraph_t graph = nullptr;
  int st = cuda_status(cudaStreamEndCapture(cs, &graph), "cudaStreamEndCapture");
  auto* G = new ojx_graph_s();
  G->device = cap.device;
  G->graph = graph;
  G->owned = std::move(cap.owned);
  if (!st) st = order_nodes(graph, G->order);
  if (!st) st = cuda_status(cudaGraphInstantiate(&G->exec, graph, 0), "cudaGraphInstantiate");
  if (!st) {
    for (cudaGraphNode_t n : G->order) {
      cudaGraphNodeType t;
      if (cudaGraphNodeGetType(n, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel)
        ++G->kernel_nodes;
    }
    *out = G;
    return OJX_OK;
  }
  // Failure: the launches already queued on other streams never touch these
  // buffers (they only ran inside the capture), so they can go at once.
  if (G->exec) cudaGraphExecDestroy(G->exec);
  if (G->graph) cudaGraphDestroy(G->graph);
  free_all(G->owned);
  delete G;
  return st;
}

int ojx_graph_launch(ojx_graph g, ojx_stream s) {
  if (!g || !g->exec) return set_error(OJX_ERR_INVALID, "invalid graph");
  int st = cuda_status(cudaGraphLaunch(g->exec, static_cast<cudaStream_t>(s)), "cudaGraphLaunch");
  if (!st) g_launches.fetch_add(static_cast<uint64_t>(g->kernel_nodes));
  return st;
}

int ojx_graph_destroy(ojx_graph g) {
  if (!g) return OJX_OK;
  int prev = 0;
  cudaGetDevice(&prev);
  if (prev != g->device) cudaSetDevice(g->device);
  int st = OJX_OK;
  if (!g->owned.empty())  // replays still in flight may use the owned buffers
    st = cuda_status(cudaDeviceSynchronize(), "graph destroy: device sync");
  if (g->exec) cudaGraphExecDestroy(g->exec);
  if (g->graph) cudaGraphDestroy(g->graph);
  free_all(g->owned);
  if (prev != g->device) cudaSetDevice(prev);
  delete g;
  return st;
}

int ojx_graph_node_count(ojx_graph g, int kernels_only, int32_t* n) {
  if (!g || !n) return set_error(OJX_ERR_INVALID, "invalid graph or NULL out");
  *n = kernels_only ? g->kernel_nodes : static_cast<int32_t>(g->order.size());
  return OJX_OK;
}

int ojx_graph_node_get(ojx_graph g, int32_t index, ojx_graph_node* out) {
  if (!g || !out) return set_error(OJX_ERR_INVALID, "invalid graph or NULL out");
  if (index < 0 || static_cast<size_t>(index) >= g->order.size())
    return set_error(OJX_ERR_INVALID, "node index %d out of range [0, %zu)", index, g->order.size());
  std::memset(out, 0, sizeof(*out));
  cudaGraphNode_t n = g->order[static_cast<size_t>(index)];
  cudaGraphNodeType t;
  if (int st = cuda_status(cudaGraphNodeGetType(n, &t), "cudaGraphNodeGetType")) return st;
  if (t == cudaGraphNodeTypeKernel) {
    cudaKernelNodeParams kp{};
    if (int st = cuda_status(cudaGraphKernelNodeGetParams(n, &kp), "cudaGraphKernelNodeGetParams"))
      return st;
    out->type = OJX_NODE_KERNEL;
    out->grid[0] = static_cast<int32_t>(kp.gridDim.x);
    out->grid[1] = static_cast<int32_t>(kp.gridDim.y);
    out->grid[2] = static_cast<int32_t>(kp.gridDim.z);
    out->block[0] = static_cast<int32_t>(kp.blockDim.x);
    out->block[1] = static_cast<int32_t>(kp.blockDim.y);
    out->block[2] = static_cast<int32_t>(kp.blockDim.z);
    out->smem_bytes = static_cast<int32_t>(kp.sharedMemBytes);
    const char* name = nullptr;
    if (cudaFuncGetName(&name, kp.func) == cudaSuccess)
      short_name(name, out->name, sizeof(out->name));
    else
      (void)cudaGetLastError();
  } else if (t == cudaGraphNodeTypeMemset) {
    out->type = OJX_NODE_MEMSET;
    std::snprintf(out->name, sizeof(out->name), "memset");
  } else if (t == cudaGraphNodeTypeMemcpy) {
    out->type = OJX_NODE_MEMCPY;
    std::snprintf(out->name, sizeof(out->name), "memcpy");
  } else {
    out->type = OJX_NODE_OTHER;
  }
  return OJX_OK;
}

}  // extern "C"
