"""Layer steps over batches in pinned host memory, copies overlapped with compute.

A serving loop feeds the MoE layer one batch of hidden states after another
from host memory and reads each result back.  ``HostPipeline`` keeps two
device slots: while the layer (one CUDA graph per slot) runs on batch i, the
copy engines upload batch i+1 and download batch i-1 on their own streams, so
a step costs max(upload, layer, download) instead of their sum.  Every batch
is still copied in and out in full; events order the three streams:

  upload i   waits for the layer step that last read slot i % 2 (batch i-2);
  layer i    waits for upload i and for the download of batch i-2 (the last
             reader of the slot's output);
  download i waits for layer i.

The layer is anything callable on a bf16 device tensor [T, H] that returns
[T, H]: ``MoELayer``, ``HashMoELayer`` without token ids, or a peer-exchange
``ExpertParallelMoELayer`` (whose step is graph-capturable).
"""
from __future__ import annotations

import os

import torch


def gpu_numa_cpus(device_index: int) -> set | None:
    """The CPUs of the NUMA node the GPU's PCI device hangs off (Linux sysfs),
    or None when that is unknown.  A process that binds to them
    (``os.sched_setaffinity``) before pinning host memory gets its pinned
    buffers on the GPU's node, so several GPUs' uploads and downloads do not
    cross the socket interconnect."""
    try:
        p = torch.cuda.get_device_properties(device_index)
        bus = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        with open(f"/sys/bus/pci/devices/{bus}/numa_node") as f:
            node = int(f.read().strip())
        if node < 0:
            return None
        with open(f"/sys/devices/system/node/node{node}/cpulist") as f:
            spec = f.read().strip()
        cpus = set()
        for part in spec.split(","):
            if "-" in part:
                a, b = part.split("-")
                cpus.update(range(int(a), int(b) + 1))
            elif part:
                cpus.add(int(part))
        return cpus & os.sched_getaffinity(0) or None
    except (OSError, ValueError, AttributeError, RuntimeError):
        return None


class HostPipeline:
    """Runs ``layer`` over host batches of ``tokens`` x ``hidden`` bf16 values.

    ``graph=True`` captures the layer step once per slot (the step must be
    capturable: no host synchronisation inside); ``graph=False`` launches it
    eagerly on the compute stream.
    """

    def __init__(self, layer, tokens: int, hidden: int, *, device=None, graph: bool = True):
        self.layer = layer
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.shape = (tokens, hidden)
        self.graph = graph
        self._up = torch.cuda.Stream(self.device)
        self._down = torch.cuda.Stream(self.device)
        self._x = [torch.zeros(self.shape, dtype=torch.bfloat16, device=self.device) for _ in range(2)]
        self._y = [None, None]
        self._g = [None, None]
        self._read = [None, None]   # layer step that last read slot s's input
        self._freed = [None, None]  # download that last read slot s's output
        if graph:
            with torch.cuda.device(self.device):
                for _ in range(3):  # warm-up outside capture: workspaces and library state
                    self.layer(self._x[0])
                torch.cuda.synchronize(self.device)
                for s in range(2):
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g):
                        self._y[s] = self.layer(self._x[s])
                    self._g[s] = g

    def _step(self, s: int) -> torch.Tensor:
        if self.graph:
            self._g[s].replay()
            return self._y[s]
        return self.layer(self._x[s])

    def run(self, xs_host, ys_host) -> None:
        """Layer outputs of the host batches ``xs_host`` into ``ys_host`` (pinned
        bf16 tensors of the pipeline's shape; a batch may repeat).  Returns once
        the work is queued; the caller synchronises (or records an event on the
        current stream, which waits for the last download)."""
        if len(xs_host) != len(ys_host):
            raise ValueError("one output buffer per input batch")
        for xh, yh in zip(xs_host, ys_host):
            for t in (xh, yh):
                if tuple(t.shape) != self.shape or t.dtype != torch.bfloat16 or t.device.type != "cpu":
                    raise ValueError(f"host batches must be bf16 CPU tensors of shape {self.shape}")
                if not t.is_pinned():
                    raise ValueError("host batches must be in pinned memory (tensor.pin_memory())")
        main = torch.cuda.current_stream(self.device)
        self._up.wait_stream(main)
        self._down.wait_stream(main)
        for i, (xh, yh) in enumerate(zip(xs_host, ys_host)):
            s = i & 1
            with torch.cuda.stream(self._up):
                if self._read[s] is not None:
                    self._up.wait_event(self._read[s])
                self._x[s].copy_(xh, non_blocking=True)
                loaded = torch.cuda.Event()
                loaded.record(self._up)
            main.wait_event(loaded)
            if self._freed[s] is not None:
                main.wait_event(self._freed[s])
            y = self._step(s)
            done = torch.cuda.Event()
            done.record(main)
            self._read[s] = done
            with torch.cuda.stream(self._down):
                self._down.wait_event(done)
                yh.copy_(y, non_blocking=True)
                freed = torch.cuda.Event()
                freed.record(self._down)
            self._freed[s] = freed
            if not self.graph:
                y.record_stream(self._down)  # the allocator keeps it until its download ran
                self._y[s] = y
        main.wait_stream(self._up)
        main.wait_stream(self._down)

    def close(self) -> None:
        """Releases the graphs (before a process group that their steps use is destroyed)."""
        torch.cuda.synchronize(self.device)
        self._g = [None, None]
        self._y = [None, None]
