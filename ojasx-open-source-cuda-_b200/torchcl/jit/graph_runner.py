"""Graph capture and replay — replaces torchcl/jit/graph_runner.py.

Same surface: `capture_graph(name)` is a context manager yielding a
`CapturedGraph`; `CapturedGraph.replay(queue=None)` re-runs what was recorded,
`len(graph)` / `graph.commands` list the recorded kernel launches
(`RecordedCommand(kernel, global_size, local_size, args)`), and
`get_active_capture_graph()` returns the graph being recorded.

How it differs underneath (graph_runner.py:35-90 keeps a Python list of pyopencl
calls and re-issues them one by one):
  * the `with` block runs on a fresh stream under a CUDA stream capture
    (ojx_graph_capture_begin); every library launch made inside it is recorded,
    and one cudaGraphLaunch replays the whole sequence;
  * lazy GEMM / elementwise nodes created inside the block and still alive at its
    end are materialised before the capture closes, so the fused GEMM epilogues
    are part of the graph;
  * when the block ends the graph runs once, so its outputs hold values just as
    the reference's (which executes while recording);
  * nothing executes during the block: uploads (`to_opencl`), downloads
    (`to_cpu`) and `synchronize()` raise there.  Upload inputs before the block;
  * buffers used by the graph stay reserved until the graph is closed (or
    garbage collected), even if their tensors are freed.
Replays re-read the same input buffers and overwrite the same output buffers;
refresh inputs in place (e.g. `runtime.memory` host_to_device into the existing
buffer) between replays.  After a device error (OJX_ERR_TIMEOUT) capture again.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Any, List, Optional, Tuple

from torchcl import _lib as L
from torchcl.runtime import memory as _mem
from torchcl.runtime.context import _ensure_initialized, _set_current_queue, get_queue


@dataclass
class RecordedCommand:
    """One recorded launch (graph_runner.py:25-32).  For launches captured from the
    library, `kernel` is the kernel's name, `global_size` = grid x block threads
    and `local_size` = block; `args` is empty (the arguments live in the graph)."""
    kernel: Any
    global_size: Tuple[int, ...]
    local_size: Optional[Tuple[int, ...]]
    args: List[Any] = field(default_factory=list)


class CapturedGraph:
    """A recorded launch sequence ready for replay (graph_runner.py:35-65)."""

    def __init__(self, name: str = "captured_graph") -> None:
        self.name = name
        self.commands: List[RecordedCommand] = []
        self._graph: int | None = None
        self._pinned: list[int] = []
        self._host_commands: List[RecordedCommand] = []

    # The reference's engine calls this for every launch while recording.  Here
    # the stream capture records library launches by itself; commands added
    # through this method (a callable `kernel(queue, global_size, local_size,
    # *args)`) are listed too and re-issued from the host after the graph on
    # every replay.
    def record_kernel_launch(self, kernel: Any, global_size: Tuple[int, ...],
                             local_size: Optional[Tuple[int, ...]], *args: Any) -> None:
        cmd = RecordedCommand(kernel=kernel, global_size=tuple(global_size),
                              local_size=None if local_size is None else tuple(local_size),
                              args=list(args))
        self.commands.append(cmd)
        self._host_commands.append(cmd)

    def _attach(self, graph: int, pinned: list[int]) -> None:
        self._graph = graph
        self._pinned = pinned
        lib = L.lib()
        n = ctypes.c_int32()
        L.check(lib.ojx_graph_node_count(graph, 0, ctypes.byref(n)), "graph nodes")
        node = L.GraphNode()
        recorded = []
        for i in range(n.value):
            L.check(lib.ojx_graph_node_get(graph, i, ctypes.byref(node)), "graph node")
            if node.type != 1:
                continue
            grid = tuple(int(x) for x in node.grid)
            block = tuple(int(x) for x in node.block)
            recorded.append(RecordedCommand(
                kernel=node.name.decode(errors="replace"),
                global_size=tuple(g * b for g, b in zip(grid, block)), local_size=block))
        self.commands = recorded + self.commands

    def replay(self, queue: Optional[int] = None) -> None:
        """Launch the recorded sequence on `queue` (default: the current stream)."""
        if self._graph is None and not self._host_commands:
            return
        q = queue if queue is not None else get_queue()
        if self._graph is not None:
            L.check(L.lib().ojx_graph_launch(self._graph, q), "graph replay")
        for cmd in self._host_commands:
            cmd.kernel(q, cmd.global_size, cmd.local_size, *cmd.args)

    def close(self) -> None:
        """Free the CUDA graph and release the buffers it kept reserved."""
        g, self._graph = self._graph, None
        if g is not None:
            L.check(L.lib().ojx_graph_destroy(g), "graph destroy")
        pins, self._pinned = self._pinned, []
        if pins:
            _mem.release_pins(pins)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __len__(self) -> int:
        return len(self.commands)


_active_capture_graph: Optional[CapturedGraph] = None


class capture_graph:
    """Context manager recording library launches into a CapturedGraph (graph_runner.py:70-86)."""

    def __init__(self, name: str = "captured_graph") -> None:
        self.graph = CapturedGraph(name=name)
        self._stream = None
        self._prev_queue = None

    def __enter__(self) -> CapturedGraph:
        global _active_capture_graph
        if _active_capture_graph is not None:
            raise RuntimeError("capture_graph blocks do not nest")
        _ensure_initialized()
        from torchcl import api
        from torchcl.runtime.stream import Stream
        self._prev_queue = get_queue()
        self._stream = Stream()
        _mem.begin_capture()
        try:
            L.check(L.lib().ojx_graph_capture_begin(self._stream.queue), "graph capture")
        except Exception:
            _mem.end_capture(keep=False)
            raise
        api._capture_lazy = []
        _set_current_queue(self._stream.queue)
        _active_capture_graph = self.graph
        return self.graph

    def __exit__(self, exc_type, exc_val, exc_tb) -> bool:
        global _active_capture_graph
        from torchcl import api
        err = None
        try:
            if exc_type is None:
                for ref in api._capture_lazy or []:
                    h = ref()
                    if h is not None and api._is_lazy(h):
                        api.materialize_lazy_tensor(h)
        except Exception as e:  # the capture must still be closed
            err = e
        finally:
            api._capture_lazy = None
            _set_current_queue(self._prev_queue)
            _active_capture_graph = None
            g = ctypes.c_void_p()
            rc = L.lib().ojx_graph_capture_end(self._stream.queue, ctypes.byref(g))
            msg = L.last_error() if rc else ""
            ok = rc == L.OJX_OK and exc_type is None and err is None
            pinned = _mem.end_capture(keep=rc == L.OJX_OK)
        if rc == L.OJX_OK:
            self.graph._attach(g.value, pinned)
        if exc_type is not None:
            self.graph.close()
            return False
        if err is not None:
            self.graph.close()
            raise err
        if rc != L.OJX_OK:
            raise RuntimeError(f"graph capture: {msg}")
        if ok:
            self.graph.replay(self._prev_queue)
        return False


def get_active_capture_graph() -> Optional[CapturedGraph]:
    """The graph being recorded, if any (graph_runner.py:88-90)."""
    return _active_capture_graph
