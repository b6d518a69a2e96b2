"""A stack of gated GPT-NeoX MLP layers on one GPU, with a host-to-host forward
that overlaps PCIe copies with compute.

``MLPStack`` chains layers through GPT-NeoX's parallel residual,
``x_{l+1} = round(x_l + MLP_l(x_l))`` (the MLP branch of GPTNeoXLayer.forward,
transformers/models/gpt_neox/modeling_gpt_neox.py), which the down-projection
kernel fuses.  The MLP is token-local, so tokens can be processed in independent
chunks with results identical to one pass.

``forward_host`` takes pinned host tensors of one batch: chunk i's host-to-device
copy, chunk i-1's compute and chunk i-2's device-to-host copy run on three
streams at once.  The whole schedule (copies, 2 kernels per layer per chunk,
events) is captured once into a CUDA graph per (input, output) buffer pair and
replayed, so each call costs one graph launch on the host.

``stream_host`` serves a sequence of batches: batch i+1's host-to-device copy and
batch i-1's device-to-host copy overlap batch i's compute, which runs on the whole
batch (full-size kernels) from double-buffered device slots, as a replayed graph.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops
from .gates import resolve


@dataclass
class Layer:
    w_in: torch.Tensor   # [F, d]
    b_in: torch.Tensor | None
    w_out: torch.Tensor  # [d, F]
    b_out: torch.Tensor | None
    gate: object         # gate spec mapping / module / GateSpec


class MLPStack:
    """Gated MLP layers chained by the parallel residual, resident on one CUDA device."""

    def __init__(self, layers: list[Layer], *, skip: bool | str = True):
        if not layers:
            raise ValueError("need at least one layer")
        self.layers = [Layer(L.w_in, L.b_in, L.w_out, L.b_out, resolve(L.gate)) for L in layers]
        w = self.layers[0].w_in
        self.device, self.dtype = w.device, w.dtype
        self.d, self.F = w.shape[1], w.shape[0]
        self.skip = skip
        self._ws: dict[int, tuple] = {}
        self._graphs: dict[tuple, tuple] = {}

    def _workspace(self, tokens: int):
        ws = self._ws.get(tokens)
        if ws is None:
            h = torch.empty(tokens, self.F, device=self.device, dtype=self.dtype)
            bits = torch.empty(ops.tile_bits_size(tokens, self.F), device=self.device, dtype=torch.int32)
            ping = torch.empty(tokens, self.d, device=self.device, dtype=self.dtype)
            pong = torch.empty(tokens, self.d, device=self.device, dtype=self.dtype)
            ws = self._ws[tokens] = (h, bits, ping, pong)
        return ws

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """Device forward of all layers on x [T, d]; returns out (or a workspace buffer)."""
        t = x.shape[0]
        h, bits, ping, pong = self._workspace(t)
        cur = x
        for i, L in enumerate(self.layers):
            last = i == len(self.layers) - 1
            dst = out if (last and out is not None) else (ping if cur is not ping else pong)
            ops.up_gate(cur, L.w_in, L.b_in, L.gate, h=h, bits=bits)
            ops.down_sparse(h, bits, L.w_out, L.b_out, cur, skip=self.skip, y=dst)
            cur = dst
        return cur

    # ------------------------------------------------------------ host to host
    def _schedule(self, x_host, y_host, x_dev, y_dev, chunks, streams):
        s_in, s_comp, s_out = streams
        main = torch.cuda.current_stream(self.device)
        start = torch.cuda.Event()
        start.record(main)
        for s in streams:
            s.wait_event(start)
        t = x_host.shape[0]
        bounds = [(t * c // chunks, t * (c + 1) // chunks) for c in range(chunks)]
        done = []
        for c, (lo, hi) in enumerate(bounds):
            ev_in, ev_comp, ev_out = torch.cuda.Event(), torch.cuda.Event(), torch.cuda.Event()
            with torch.cuda.stream(s_in):
                x_dev[lo:hi].copy_(x_host[lo:hi], non_blocking=True)
                ev_in.record(s_in)
            with torch.cuda.stream(s_comp):
                s_comp.wait_event(ev_in)
                self.forward(x_dev[lo:hi], out=y_dev[lo:hi])
                ev_comp.record(s_comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_comp)
                y_host[lo:hi].copy_(y_dev[lo:hi], non_blocking=True)
                ev_out.record(s_out)
            done.append(ev_out)
        for s in streams:
            ev = torch.cuda.Event()
            ev.record(s)
            main.wait_event(ev)

    def forward_host(self, x_host: torch.Tensor, y_host: torch.Tensor, *, chunks: int = 4,
                     graph: bool = True) -> torch.Tensor:
        """y_host = stack(x_host) for pinned host tensors [T, d], copies overlapped with compute.

        With ``graph`` the schedule is captured once for this buffer pair and replayed."""
        if x_host.is_cuda or y_host.is_cuda:
            raise ValueError("forward_host takes host tensors")
        if not (x_host.is_pinned() and y_host.is_pinned()):
            raise ValueError("host tensors must be pinned (tensor.pin_memory())")
        t = x_host.shape[0]
        if t % chunks:
            raise ValueError("T must divide into the chunks evenly")
        key = (x_host.data_ptr(), y_host.data_ptr(), t, chunks)
        entry = self._graphs.get(key)
        if entry is None:
            x_dev = torch.empty(t, self.d, device=self.device, dtype=self.dtype)
            y_dev = torch.empty(t, self.d, device=self.device, dtype=self.dtype)
            streams = tuple(torch.cuda.Stream(self.device) for _ in range(3))
            self._workspace(t // chunks)
            # One eager run: resolves lazy set-up (tensor-map encoder, occupancy query) outside capture.
            self._schedule(x_host, y_host, x_dev, y_dev, chunks, streams)
            torch.cuda.synchronize(self.device)
            g = None
            if graph:
                g = torch.cuda.CUDAGraph()
                side = torch.cuda.Stream(self.device)
                side.wait_stream(torch.cuda.current_stream(self.device))
                with torch.cuda.stream(side):
                    with torch.cuda.graph(g, stream=side):
                        self._schedule(x_host, y_host, x_dev, y_dev, chunks, streams)
                torch.cuda.current_stream(self.device).wait_stream(side)
            entry = self._graphs[key] = (g, x_dev, y_dev, streams)
            if g is None:
                return y_host
        g, x_dev, y_dev, streams = entry
        if g is not None:
            g.replay()
        else:
            self._schedule(x_host, y_host, x_dev, y_dev, chunks, streams)
        return y_host

    def _slots(self, tokens: int, graph: bool):
        key = ("slots", tokens, graph)
        entry = self._graphs.get(key)
        if entry is None:
            streams = tuple(torch.cuda.Stream(self.device) for _ in range(3))
            slots = []
            for _ in range(2):
                x_dev = torch.empty(tokens, self.d, device=self.device, dtype=self.dtype)
                y_dev = torch.empty(tokens, self.d, device=self.device, dtype=self.dtype)
                g = None
                if graph:
                    self.forward(x_dev, out=y_dev)  # eager run: lazy set-up happens outside capture
                    torch.cuda.synchronize(self.device)
                    g = torch.cuda.CUDAGraph()
                    side = torch.cuda.Stream(self.device)
                    side.wait_stream(torch.cuda.current_stream(self.device))
                    with torch.cuda.stream(side):
                        with torch.cuda.graph(g, stream=side):
                            self.forward(x_dev, out=y_dev)
                    torch.cuda.current_stream(self.device).wait_stream(side)
                slots.append({"x": x_dev, "y": y_dev, "graph": g, "comp_done": None, "out_done": None})
            entry = self._graphs[key] = (streams, slots)
        return entry

    def stream_host(self, x_hosts: list[torch.Tensor], y_hosts: list[torch.Tensor], *,
                    graph: bool = True) -> list[torch.Tensor]:
        """Run the stack on each pinned host batch x_hosts[i] -> y_hosts[i].

        Work is enqueued asynchronously on the current device; the current stream
        waits for all of it, so synchronising that stream (or the device) makes
        every y_hosts[i] ready."""
        if len(x_hosts) != len(y_hosts) or not x_hosts:
            raise ValueError("need matching, non-empty lists of host batches")
        t = x_hosts[0].shape[0]
        for xh, yh in zip(x_hosts, y_hosts):
            if xh.is_cuda or yh.is_cuda or not (xh.is_pinned() and yh.is_pinned()):
                raise ValueError("batches must be pinned host tensors")
            if xh.shape != (t, self.d) or yh.shape != (t, self.d):
                raise ValueError("every batch must have the same [T, d] shape")
        (s_in, s_comp, s_out), slots = self._slots(t, graph)
        main = torch.cuda.current_stream(self.device)
        start = torch.cuda.Event()
        start.record(main)
        for st in (s_in, s_comp, s_out):
            st.wait_event(start)
        for i, (xh, yh) in enumerate(zip(x_hosts, y_hosts)):
            sl = slots[i % 2]
            in_done, comp_done, out_done = torch.cuda.Event(), torch.cuda.Event(), torch.cuda.Event()
            with torch.cuda.stream(s_in):
                if sl["comp_done"] is not None:
                    s_in.wait_event(sl["comp_done"])  # batch i-2 no longer reads this input slot
                sl["x"].copy_(xh, non_blocking=True)
                in_done.record(s_in)
            with torch.cuda.stream(s_comp):
                s_comp.wait_event(in_done)
                if sl["out_done"] is not None:
                    s_comp.wait_event(sl["out_done"])  # batch i-2's result has left this output slot
                if sl["graph"] is not None:
                    sl["graph"].replay()
                else:
                    self.forward(sl["x"], out=sl["y"])
                comp_done.record(s_comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(comp_done)
                yh.copy_(sl["y"], non_blocking=True)
                out_done.record(s_out)
            sl["comp_done"], sl["out_done"] = comp_done, out_done
        for st in (s_in, s_comp, s_out):
            ev = torch.cuda.Event()
            ev.record(st)
            main.wait_event(ev)
        return y_hosts
