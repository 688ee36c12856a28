#!/usr/bin/env python3
"""Benchmark of the Mote Q4_0 / per-token layer data plane on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline (BASELINE metric "Q4_0 decode-linear HBM GB/s vs 8 TB/s peak; fused
RMSNorm+RoPE us/layer"): one step is one pass of the config-3 batch-decode
sweep -- Q4_0 linear with M in {1,2,4,8,16}, K=4096, N in {4096,11008,14336},
f16 activations, f32 accumulation, f16 output -- where every (M, N) case
runs once over each of R_N rotating copies of its weight matrix.  R_N copies
hold >= 2.5x the 126 MB L2, so every launch streams its weights from HBM
("inputs larger than L2").  value = algorithmic bytes (Q4_0 weights once +
activations + outputs) per second over all ranks.  The step is captured in a
CUDA graph and timed with CUDA events; multi-GPU runs are independent
replicas (weak scaling) timed as the max over ranks.

Extra figures in the same JSON line: config 1 (f32 M=1 K=N=2048), config 2
(fused RMSNorm + RoPE, us per layer), config 5 (lm_head K=4096 N=128256 at
M in {1,16,64}; prefill M=2048 TFLOP/s), and at N>1 the column-sharded
lm_head with an NCCL all-gather of the f16 outputs.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "Q4_0 decode-linear HBM GB/s vs 8 TB/s peak; fused RMSNorm+RoPE µs/layer"
SPEC_HBM_GBS = 8000.0
L2_BYTES = 126 * 1024 * 1024
ROTATION_BYTES = int(2.5 * L2_BYTES)
SWEEP_M = (1, 2, 4, 8, 16)
SWEEP_N = (4096, 11008, 14336)
SWEEP_K = 4096


def q4_bytes(n: int, k: int) -> int:
    return n * (k // 32) * 18


def linear_bytes(m: int, n: int, k: int, in_size: int = 2, out_size: int = 2) -> int:
    """Algorithmic bytes of one Q4_0 linear: weights once + x + y."""
    return q4_bytes(n, k) + m * k * in_size + m * n * out_size


def copies_for(nbytes: int) -> int:
    return max(1, math.ceil(ROTATION_BYTES / nbytes))


# --------------------------------------------------------------------------
def measured_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.device_index), "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (FileNotFoundError, OSError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------------------
class Bench:
    def __init__(self, args):
        import torch

        self.args = args
        self.torch = torch
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local_rank)
        self.dev = torch.device("cuda", self.local_rank)
        # The C ABI (like the reference shim) rejects the null stream, which is
        # torch's default stream handle: run everything on an explicit stream.
        self.main_stream = torch.cuda.Stream(device=self.dev)
        torch.cuda.set_stream(self.main_stream)
        from mote_b200 import _native

        self.lib = _native.lib()
        assert self.lib.mote_cuda_set_device(self.local_rank) == 0
        self.launches = 0
        if self.world > 1:
            import datetime

            # plain NVLink transports only: no NVLink multicast objects
            os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
            torch.distributed.init_process_group(
                "nccl", timeout=datetime.timedelta(seconds=120),
                device_id=self.dev)

    # -- helpers -----------------------------------------------------------
    def stream(self) -> int:
        return self.torch.cuda.current_stream().cuda_stream

    def check(self, status: int, what: str):
        if status != 0:
            from mote_b200._native import status_string

            raise RuntimeError(f"{what}: status {status} ({status_string(status)})")

    def encode_into(self, ptr: int, n: int, k: int, seed: int) -> None:
        """W ~ N(0, 0.02) generated on device, Q4_0-encoded by our encoder into ptr."""
        torch = self.torch
        g = torch.Generator(device=self.dev).manual_seed(seed)
        rows_per = max(1, (256 << 20) // (k * 4))
        for r0 in range(0, n, rows_per):
            r1 = min(n, r0 + rows_per)
            f = torch.randn((r1 - r0, k), generator=g, device=self.dev, dtype=torch.float32)
            f.mul_(0.02)
            self.check(self.lib.mote_cuda_q4_0_encode_f32(
                f.data_ptr(), ptr + r0 * (k // 32) * 18, r1 - r0, k, self.stream()), "encode")
        torch.cuda.synchronize()

    def encode_q4_0(self, n: int, k: int, seed: int):
        w = self.torch.empty(q4_bytes(n, k), dtype=self.torch.uint8, device=self.dev)
        self.encode_into(w.data_ptr(), n, k, seed)
        return w

    def randn(self, shape, seed, dtype, scale=1.0, shift=0.0):
        torch = self.torch
        g = torch.Generator(device=self.dev).manual_seed(seed)
        t = torch.randn(shape, generator=g, device=self.dev, dtype=torch.float32)
        return (t * scale + shift).to(dtype)

    def graph(self, fn):
        torch = self.torch
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            fn()  # warm-up launch outside capture (sets kernel attributes)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        torch.cuda.synchronize()
        return g

    def time_graph(self, g, reps: int, launches_per_replay: int) -> float:
        """Average ms per replay over `reps` replays (events on the stream)."""
        torch = self.torch
        for _ in range(2):
            g.replay()
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(reps):
            g.replay()
        end.record()
        end.synchronize()
        self.launches += reps * launches_per_replay
        return start.elapsed_time(end) / reps

    def max_over_ranks(self, value: float) -> float:
        if self.world == 1:
            return value
        t = self.torch.tensor([value], device=self.dev, dtype=self.torch.float64)
        self.torch.distributed.all_reduce(t, op=self.torch.distributed.ReduceOp.MAX)
        return float(t.item())

    def barrier(self):
        if self.world > 1:
            self.torch.distributed.barrier(device_ids=[self.local_rank])
        self.torch.cuda.synchronize()

    # -- config 3 sweep (headline) ------------------------------------------
    def build_sweep(self):
        torch = self.torch
        k = SWEEP_K
        self.sweep_w = {}
        for n in SWEEP_N:
            r = copies_for(q4_bytes(n, k))
            base = self.encode_q4_0(n, k, seed=1000 + n)
            self.sweep_w[n] = [base] + [base.clone() for _ in range(r - 1)]
        self.sweep_x = {m: self.randn((m, k), 77 + m, torch.float16) for m in SWEEP_M}
        self.sweep_y = {(m, n): torch.empty((m, n), dtype=torch.float16, device=self.dev)
                        for m in SWEEP_M for n in SWEEP_N}
        # one zeroed workspace for the split-K path (its counters return to
        # zero after every call; the sweep runs on one stream)
        need = max(self.workspace_bytes(m, n, k) for m in SWEEP_M for n in SWEEP_N)
        self.workspace = torch.zeros(max(need, 256), dtype=torch.uint8, device=self.dev)
        self.sweep_launches = sum(len(self.sweep_w[n]) for n in SWEEP_N) * len(SWEEP_M)
        self.sweep_bytes = sum(linear_bytes(m, n, k) * len(self.sweep_w[n])
                               for m in SWEEP_M for n in SWEEP_N)

    def workspace_bytes(self, m, n, k) -> int:
        need = ctypes.c_uint64(0)
        self.check(self.lib.mote_cuda_q4_0_linear_workspace_bytes(m, n, k, ctypes.byref(need)),
                   "workspace size")
        return need.value

    def sweep_case(self, m, n):
        fn = self.lib.mote_cuda_quantized_linear_q4_0_f16_ws
        x, y = self.sweep_x[m], self.sweep_y[(m, n)]
        ws = self.workspace
        for w in self.sweep_w[n]:
            self.check(fn(x.data_ptr(), w.data_ptr(), y.data_ptr(), m, n, SWEEP_K, ws.data_ptr(),
                          ws.numel(), self.stream()), "q4_0 linear")

    def sweep_step(self):
        for m in SWEEP_M:
            for n in SWEEP_N:
                self.sweep_case(m, n)

    # -- public-API end-to-end leg ------------------------------------------------
    def e2e(self, steps: int, early: int = 2) -> dict:
        """Config-3 sweep with host buffers through the C ABI the reference's
        Rust crate binds (include/mote_cuda.h, called here through ctypes
        with the arguments prepared once, as a Rust caller holds them).  The
        five activation matrices sit in one pinned host buffer and one device
        arena, the 15 outputs likewise (16-byte aligned offsets, as the ABI
        requires).  Every step copies the activations up in one copy and runs
        the 15 linears back to back (the workspace entry, as mote_b200.ops
        calls it), the token counts largest first.  The outputs of the first
        ``early`` token counts go down on a second stream, ordered after
        their linears by an event, while the later linears run; the rest go
        down in one copy at the end; then both streams are synchronized.
        (An event between two linears breaks their programmatic dependent
        launch, so only the largest outputs are worth one.)"""
        import numpy as np

        from mote_b200.context import CudaContext, PinnedBuffer
        from mote_b200.types import DType, plain, quantized

        ctx = CudaContext(self.local_rank)
        lib = self.lib
        k = SWEEP_K
        order = sorted(SWEEP_M, reverse=True)
        # each step takes the next of R_N copies of every weight matrix (the
        # copies of one N hold >= 2.5x L2), so every step streams from HBM
        weights = {}
        for n in SWEEP_N:
            weights[n] = []
            for _ in range(copies_for(q4_bytes(n, k))):
                wt = ctx.empty(quantized((n, k)))
                self.encode_into(wt.pointer, n, k, seed=1000 + n)
                weights[n].append(wt)
        x_off, off = {}, 0
        for m in order:
            x_off[m] = off
            off += m * k * 2
        h2d = off
        y_off, y_group, off = {}, {}, 0
        for m in order:
            start = off
            for n in SWEEP_N:
                y_off[(m, n)] = off
                off += m * n * 2
            y_group[m] = (start, off - start)
        d2h = off
        assert all(v % 16 == 0 for v in list(x_off.values()) + list(y_off.values()))
        x_dev = ctx.empty(plain((h2d // 2,), DType.F16))
        y_dev = ctx.empty(plain((d2h // 2,), DType.F16))
        hx, hy = PinnedBuffer(h2d), PinnedBuffer(d2h)
        hx.view(np.float16)[:] = np.random.default_rng(5).normal(0, 1, h2d // 2).astype(np.float16)
        alg = sum(linear_bytes(m, n, k) for m in SWEEP_M for n in SWEEP_N)
        need = max(ctx.linear_workspace_bytes(m, n, k) for m in SWEEP_M for n in SWEEP_N)
        ws_ptr, ws_bytes = ctx.linear_workspace(need)
        stream = ctx.stream
        copy_stream, event = ctx.inner.copy_channel()
        groups = [(m, [(x_dev.pointer + x_off[m], [w.pointer for w in weights[n]],
                        y_dev.pointer + y_off[(m, n)], n) for n in SWEEP_N],
                   gi < early, y_group[m]) for gi, m in enumerate(order)]
        tail = y_group[order[early]][0] if early < len(order) else d2h
        upload = lib.mote_cuda_memcpy_host_to_device_async
        linear = lib.mote_cuda_quantized_linear_q4_0_f16_ws
        download = lib.mote_cuda_memcpy_device_to_host_async
        record = lib.mote_cuda_event_record
        wait = lib.mote_cuda_stream_wait_event
        sync = lib.mote_cuda_stream_synchronize

        def step(i):
            st = upload(x_dev.pointer, hx.pointer, h2d, stream)
            for m, lins, ahead, (g0, gbytes) in groups:
                for xp, wps, yp, n in lins:
                    st |= linear(xp, wps[i % len(wps)], yp, m, n, k, ws_ptr, ws_bytes, stream)
                if ahead:
                    st |= record(event, stream)
                    st |= wait(copy_stream, event)
                    st |= download(hy.pointer + g0, y_dev.pointer + g0, gbytes, copy_stream)
            if tail < d2h:
                st |= download(hy.pointer + tail, y_dev.pointer + tail, d2h - tail, stream)
            st |= sync(stream)
            st |= sync(copy_stream)
            if st:
                raise RuntimeError(f"e2e step: CUDA status {st}")

        ctx.inner.select()
        for i in range(3):
            step(i)
        t0 = time.perf_counter()
        for i in range(steps):
            step(i)
        dt = time.perf_counter() - t0
        self.launches += steps * len(SWEEP_M) * len(SWEEP_N)
        dt = self.max_over_ranks(dt)
        return {"value": round(alg * steps * self.world / dt / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(dt * 1e3 / steps, 4),
                "path": "C ABI (include/mote_cuda.h: mote_cuda_quantized_linear_q4_0_f16_ws, "
                        "the async copies, mote_cuda_stream_wait_event) through ctypes; per "
                        "step: the activations H2D from pinned host memory in one copy, the 15 "
                        f"linears back to back (16 tokens first), the outputs of the first "
                        f"{early} token counts D2H on a second stream while the later linears "
                        "run, the rest in one copy, both streams synchronized; weights rotated "
                        "over copies holding >= 2.5x L2 per N"}

    # -- extra configs ----------------------------------------------------------
    def config1(self) -> dict:
        torch = self.torch
        m, n, k = 1, 2048, 2048
        base = self.encode_q4_0(n, k, seed=1)
        r = copies_for(q4_bytes(n, k))
        ws = [base] + [base.clone() for _ in range(r - 1)]
        x = self.randn((m, k), 2, torch.float32)
        y = torch.empty((m, n), dtype=torch.float32, device=self.dev)
        fn = self.lib.mote_cuda_quantized_linear_q4_0_f32

        def run():
            for w in ws:
                self.check(fn(x.data_ptr(), w.data_ptr(), y.data_ptr(), m, n, k, self.stream()),
                           "config1")

        g = self.graph(run)
        ms = self.time_graph(g, 20, len(ws)) / len(ws)
        b = linear_bytes(m, n, k, 4, 4)
        del ws
        return {"us": round(ms * 1e3, 3), "gbs": round(b / ms / 1e6, 1),
                "bytes": b, "copies": r}

    def config2(self) -> dict:
        torch = self.torch
        t, hidden, qh, kh, hd = 512, 2048, 32, 8, 64
        eps = 1e-6
        nbytes = (2 * t * hidden + 2 * t * qh * hd + 2 * t * kh * hd) * 2 + hidden * 2 + \
            2 * t * (hd // 2) * 4
        r = copies_for(nbytes)
        pos = torch.arange(t, dtype=torch.int32, device=self.dev)
        cos = torch.empty((t, hd // 2), dtype=torch.float32, device=self.dev)
        sin = torch.empty_like(cos)
        self.check(self.lib.mote_cuda_rope_cos_sin_f32(pos.data_ptr(), cos.data_ptr(),
                                                       sin.data_ptr(), t, hd,
                                                       ctypes.c_double(10000.0), self.stream()),
                   "rope table")
        gamma = self.randn((hidden,), 3, torch.float16, 0.1, 1.0)
        sets = []
        for i in range(r):
            x = self.randn((t, hidden), 10 + i, torch.float16)
            q = self.randn((t, qh, hd), 1000 + i, torch.float16)
            kk = self.randn((t, kh, hd), 2000 + i, torch.float16)
            sets.append((x, torch.empty_like(x), q, torch.empty_like(q), kk, torch.empty_like(kk),
                         cos.clone(), sin.clone()))
        fn = self.lib.mote_cuda_rms_norm_rope_f16

        def run():
            for (x, xo, q, qo, kk, ko, c, s) in sets:
                self.check(fn(x.data_ptr(), gamma.data_ptr(), xo.data_ptr(), q.data_ptr(),
                              qo.data_ptr(), kk.data_ptr(), ko.data_ptr(), c.data_ptr(),
                              s.data_ptr(), t, hidden, qh, kh, hd, 0, ctypes.c_float(eps),
                              self.stream()), "norm+rope")

        g = self.graph(run)
        ms = self.time_graph(g, 20, r) / r
        del sets
        return {"us_per_layer": round(ms * 1e3, 3), "gbs": round(nbytes / ms / 1e6, 1),
                "bytes": nbytes, "copies": r}

    def torch_view(self, ptr: int, nbytes: int):
        """A uint8 torch view of device memory owned by a mote_b200 context."""
        class _Array:
            __cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1",
                                        "data": (ptr, False), "strides": None, "version": 3}

        return self.torch.as_tensor(_Array(), device=self.dev)

    def config4(self) -> dict:
        """Decoder-layer chain at M=1 (Llama-3.2-1B shapes) through
        mote_b200.decoder: a stack of layers with distinct weights holding
        >= 2.5x L2, the first gathering its input from the embedding table and
        each next one taking the previous layer's output.  One CUDA graph
        replays the whole stack; us/layer = replay time / layers."""
        torch = self.torch
        from mote_b200 import decoder
        from mote_b200.context import CudaContext
        from mote_b200.types import DType, plain, quantized

        ctx = CudaContext(self.local_rank)
        shape = decoder.LayerShape()
        hdim = shape.hidden
        per_layer = shape.weight_bytes()
        count = copies_for(per_layer)
        table = ctx.empty(plain((shape.vocab, hdim), DType.F16))
        self.torch_view(table.pointer, shape.vocab * hdim * 2).view(torch.float16).copy_(
            self.randn((shape.vocab, hdim), 400, torch.float16, 0.02).reshape(-1))
        layers = []
        for i in range(count):
            def q4(n, k, seed):
                w = ctx.empty(quantized((n, k)))
                self.encode_into(w.pointer, n, k, seed)
                return w

            gam = []
            for j in range(2):
                g = ctx.empty(plain((hdim,), DType.F16))
                self.torch_view(g.pointer, hdim * 2).view(torch.float16).copy_(
                    self.randn((hdim,), 500 + 2 * i + j, torch.float16, 0.1, 1.0))
                gam.append(g)
            s0 = 600 + 8 * i
            layer = decoder.DecoderLayerQ4_0(
                ctx, shape, embedding=table, w_qkv=q4(shape.qkv, hdim, s0),
                w_o=q4(hdim, hdim, s0 + 1), w_gate=q4(shape.ffn, hdim, s0 + 2),
                w_up=q4(shape.ffn, hdim, s0 + 3), w_down=q4(hdim, shape.ffn, s0 + 4),
                gamma1=gam[0], gamma2=gam[1])
            self.torch_view(layer.attn.pointer, hdim * 2).view(torch.float16).copy_(
                self.randn((hdim,), 700 + i, torch.float16))
            layers.append(layer)
        torch.cuda.synchronize()
        import numpy as np

        ctx.upload_numpy(layers[0].ids, np.array([1234], np.int32))
        for layer in layers:
            layer.set_position(77)

        def run_chain():
            layers[0].step()
            for prev, layer in zip(layers, layers[1:]):
                layer.step(prev.out)

        def run_fused():
            layers[0].step_fused()
            for prev, layer in zip(layers, layers[1:]):
                layer.step_fused(prev.out)

        from mote_b200 import ops

        stack = decoder.DecoderStackQ4_0(ctx, layers)

        def run_stack():
            ops.embedding_gather_f16(ctx, table, layers[0].ids, layers[0].h, check=False)
            stack.run(layers[0].h)

        result = {"weight_bytes_per_layer": per_layer, "layers_in_stack": count,
                  "bytes": "Q4_0 weight bytes of QKV, O, gate, up, down (activations < 0.3%)"}
        # kernels per layer -- chain: rms_norm, QKV, 2 x RoPE, O, fused
        # add+norm, gate/up+SwiGLU, down+residual; fused: norm+QKV+RoPE,
        # O+residual, norm+gate/up+SwiGLU, down+residual; plus one gather
        # stack: one persistent cooperative launch for all layers (plus the
        # gather and the barrier-word reset)
        for name, body, kernels in (("chain", run_chain, 8), ("fused", run_fused, 4),
                                    ("stack", run_stack, None)):
            body()
            ctx.sync()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=torch.cuda.ExternalStream(ctx.stream)):
                body()
            launches = 2 if kernels is None else kernels * count + 1
            ms = self.time_graph(g, 20, launches) / count
            assert ctx.device_status() == 0
            del g
            result[name] = {"us_per_layer": round(ms * 1e3, 3),
                            "gbs": round(per_layer / ms / 1e6, 1),
                            "kernels_per_layer": kernels if kernels else round(1 / count, 3)}
        del layers, stack
        result["us_per_layer"] = min(result[k]["us_per_layer"] for k in ("chain", "fused", "stack"))
        return result

    def config5(self) -> dict:
        torch = self.torch
        k, n = 4096, 128256
        w = self.encode_q4_0(n, k, seed=55)  # 295.5 MB > 2 x L2: no rotation needed
        out = {}
        fn = self.lib.mote_cuda_quantized_linear_q4_0_f16
        fn_ws = self.lib.mote_cuda_quantized_linear_q4_0_f16_ws
        ws = torch.zeros(max(self.workspace_bytes(16, n, k), 256), dtype=torch.uint8,
                         device=self.dev)
        for m in (1, 16, 64):
            x = self.randn((m, k), 60 + m, torch.float16)
            y = torch.empty((m, n), dtype=torch.float16, device=self.dev)

            def run(x=x, y=y, m=m):
                self.check(fn_ws(x.data_ptr(), w.data_ptr(), y.data_ptr(), m, n, k, ws.data_ptr(),
                                 ws.numel(), self.stream()), "lm_head")

            g = self.graph(run)
            ms = self.time_graph(g, 20, 1)
            b = linear_bytes(m, n, k)
            out[f"lm_head_m{m}"] = {"us": round(ms * 1e3, 2), "gbs": round(b / ms / 1e6, 1)}
        del w
        # prefill-shaped GEMM: M=2048, K=4096, N=14336
        m, n = 2048, 14336
        w = self.sweep_w[n][0]
        x = self.randn((m, k), 99, torch.float16)
        y = torch.empty((m, n), dtype=torch.float16, device=self.dev)

        wsp = torch.zeros(max(self.workspace_bytes(m, n, k), 256), dtype=torch.uint8,
                          device=self.dev)

        def runp():
            # the workspace entry (what mote_b200.ops calls): the partial last
            # wave of tiles is split along K through the workspace
            self.check(fn_ws(x.data_ptr(), w.data_ptr(), y.data_ptr(), m, n, k, wsp.data_ptr(),
                             wsp.numel(), self.stream()), "prefill")

        g = self.graph(runp)
        ms = self.time_graph(g, 5, 1)
        flops = 2.0 * m * n * k
        out["prefill_m2048"] = {"us": round(ms * 1e3, 1),
                                "tflops": round(flops / ms / 1e9, 1)}
        return out

    def q8_0(self) -> dict:
        """The Q8_0 linear (next after the Q4_0 path): lm_head K=4096,
        N=128256 at M in {1, 16} (558 MB of weights, no rotation needed) and
        N=14336 at M=1 over copies holding >= 2.5x L2.  Weights are random
        signed bytes with a fixed small f16 scale (timing only; parity is in
        tests/test_gpu_q8_0.py)."""
        torch = self.torch
        fn = self.lib.mote_cuda_quantized_linear_q8_0_f16
        k = 4096
        out = {}
        for n, ms in ((128256, (1, 16)), (14336, (1,))):
            nb = n * (k // 32) * 34
            g0 = torch.Generator(device=self.dev).manual_seed(n)
            base = torch.randint(0, 256, (nb,), generator=g0, dtype=torch.uint8, device=self.dev)
            blocks = base.view(n * (k // 32), 34)
            blocks[:, 0] = 0
            blocks[:, 1] = 0x20  # f16 scale bits 0x2000
            ws = [base] + [base.clone() for _ in range(copies_for(nb) - 1)]
            for m in ms:
                x = self.randn((m, k), 70 + m, torch.float16)
                y = torch.empty((m, n), dtype=torch.float16, device=self.dev)

                def run(x=x, y=y, m=m, n=n, ws=ws):
                    for w in ws:
                        self.check(fn(x.data_ptr(), w.data_ptr(), y.data_ptr(), m, n, k,
                                      self.stream()), "q8_0 linear")

                g = self.graph(run)
                t = self.time_graph(g, 10, len(ws)) / len(ws)
                del g
                b = nb + m * k * 2 + m * n * 2
                out[f"m{m}_n{n}"] = {"us": round(t * 1e3, 2), "gbs": round(b / t / 1e6, 1),
                                     "weight_bytes": nb, "copies": len(ws)}
            del ws, base
        return out

    def kquant_weights(self, name: str, n: int, k: int, seed: int):
        """Random K-quant super-blocks with small fixed f16 scales (timing only;
        parity is in tests/test_gpu_kquant.py)."""
        torch = self.torch
        bb = 144 if name == "q4_k" else 210
        nb = n * (k // 256) * bb
        g0 = torch.Generator(device=self.dev).manual_seed(seed)
        base = torch.randint(0, 256, (nb,), generator=g0, dtype=torch.uint8, device=self.dev)
        blocks = base.view(n * (k // 256), bb)
        if name == "q4_k":
            blocks[:, 0:4] = torch.tensor([0, 0x08, 0, 0x08], dtype=torch.uint8, device=self.dev)
        else:
            blocks[:, 208:210] = torch.tensor([0, 0x10], dtype=torch.uint8, device=self.dev)
        return base, nb

    def kquant(self) -> dict:
        """The K-quant linears (tensor-core decode kernels): lm_head K=4096,
        N=128256 at M in {1, 16} (Q4_K 295.5 MB, Q6_K 431 MB: no rotation
        needed) and N=14336 at M=1 over copies holding >= 2.5x L2; and the
        Q4_K and Q6_K prefill M=2048, N=14336 on the tcgen05 GEMM (TFLOP/s)."""
        torch = self.torch
        k = 4096
        out = {}
        for name, n, ms in (("q4_k", 128256, (1, 16)), ("q4_k", 14336, (1,)),
                            ("q6_k", 128256, (1, 16)), ("q6_k", 14336, (1,))):
            fn = getattr(self.lib, f"mote_cuda_quantized_linear_{name}_f16")
            base, nb = self.kquant_weights(name, n, k, seed=n + len(name))
            ws = [base] + [base.clone() for _ in range(copies_for(nb) - 1)]
            for m in ms:
                x = self.randn((m, k), 90 + m, torch.float16)
                y = torch.empty((m, n), dtype=torch.float16, device=self.dev)

                def run(x=x, y=y, m=m, n=n, ws=ws, fn=fn):
                    for w in ws:
                        self.check(fn(x.data_ptr(), w.data_ptr(), y.data_ptr(), m, n, k,
                                      self.stream()), "k-quant linear")

                g = self.graph(run)
                t = self.time_graph(g, 10, len(ws)) / len(ws)
                del g
                b = nb + m * k * 2 + m * n * 2
                out[f"{name}_m{m}_n{n}"] = {"us": round(t * 1e3, 2),
                                            "gbs": round(b / t / 1e6, 1),
                                            "weight_bytes": nb, "copies": len(ws)}
            del ws, base
        # Q4_K prefill on the tcgen05 GEMM (Q4_K converter): M=2048, N=14336
        m, n = 2048, 14336
        w, nb = self.kquant_weights("q4_k", n, k, seed=5)
        x = self.randn((m, k), 95, torch.float16)
        y = torch.empty((m, n), dtype=torch.float16, device=self.dev)
        fn = self.lib.mote_cuda_quantized_linear_q4_k_f16

        def runp():
            self.check(fn(x.data_ptr(), w.data_ptr(), y.data_ptr(), m, n, k, self.stream()),
                       "q4_k prefill")

        g = self.graph(runp)
        t = self.time_graph(g, 10, 1)
        del g
        out["q4_k_prefill_m2048_n14336"] = {"us": round(t * 1e3, 1),
                                             "tflops": round(2 * m * n * k / t / 1e9, 1)}
        del w
        w6, _ = self.kquant_weights("q6_k", n, k, seed=6)
        fn6 = self.lib.mote_cuda_quantized_linear_q6_k_f16

        def runp6():
            self.check(fn6(x.data_ptr(), w6.data_ptr(), y.data_ptr(), m, n, k, self.stream()),
                       "q6_k prefill")

        g = self.graph(runp6)
        t = self.time_graph(g, 10, 1)
        del g
        out["q6_k_prefill_m2048_n14336"] = {"us": round(t * 1e3, 1),
                                             "tflops": round(2 * m * n * k / t / 1e9, 1)}
        return out

    def dense_matmul(self) -> dict:
        """The dense f16 x f16 -> f32 matmul through cuBLASLt (the HIP
        backend's hipBLASLt matmul; its bench uses M=N=K in 256..2048):
        TFLOP/s at M=N=K in {1024, 2048, 4096} with a 32 MiB workspace."""
        torch = self.torch
        h = ctypes.c_void_p()
        self.check(self.lib.mote_cuda_blaslt_create(ctypes.byref(h)), "blaslt create")
        ws = torch.empty(32 << 20, dtype=torch.uint8, device=self.dev)
        out = {}
        try:
            for s_ in (1024, 2048, 4096):
                a = self.randn((s_, s_), 11, torch.float16)
                b = self.randn((s_, s_), 12, torch.float16)
                c = torch.empty((s_, s_), dtype=torch.float32, device=self.dev)

                def run(a=a, b=b, c=c, s_=s_):
                    self.check(self.lib.mote_cuda_blaslt_matmul_f16_f32(
                        h, s_, s_, s_, a.data_ptr(), b.data_ptr(), c.data_ptr(), ws.data_ptr(),
                        ws.numel(), self.stream()), "blaslt matmul")

                run()  # tunes the shape outside the graph
                torch.cuda.synchronize()
                g = self.graph(run)
                t = self.time_graph(g, 20, 1)
                del g
                out[f"mnk{s_}"] = {"us": round(t * 1e3, 1),
                                   "tflops": round(2 * s_ ** 3 / t / 1e9, 1)}
        finally:
            self.lib.mote_cuda_blaslt_destroy(h)
        return out

    def attention(self) -> dict:
        """GQA attention over a KV cache at Llama-3.2-1B geometry (32 query
        heads, 8 KV heads, head_dim 64).  Decode: one query token per
        sequence, GB/s = the K and V bytes of the attended positions (read
        once) / time, caches rotated over copies holding >= 2.5x L2.
        Prefill: causal chunks from position 0 on the tensor cores, TFLOP/s
        = 4 * head_dim * q_heads * sum over queries of attended positions."""
        torch = self.torch
        qh, kvh, hd = 32, 8, 64
        scale = ctypes.c_float(1.0 / math.sqrt(hd))
        out = {}
        for batch, length in ((1, 4096), (1, 32768), (16, 4096)):
            kv_bytes = 2 * batch * length * kvh * hd * 2
            r = copies_for(kv_bytes)
            caches = [(self.randn((batch * length, kvh, hd), 40 + i, torch.float16),
                       self.randn((batch * length, kvh, hd), 80 + i, torch.float16))
                      for i in range(r)]
            q = self.randn((batch, qh, hd), 5, torch.float16)
            o = torch.empty_like(q)
            lens = torch.full((batch,), length, dtype=torch.int32, device=self.dev)
            need = ctypes.c_uint64(0)
            self.check(self.lib.mote_cuda_gqa_attention_decode_workspace_bytes(
                batch, qh, kvh, hd, length, ctypes.byref(need)), "attention workspace")
            ws = torch.empty(max(need.value, 16), dtype=torch.uint8, device=self.dev)

            def run(caches=caches, q=q, o=o, lens=lens, ws=ws, batch=batch, length=length):
                for kc, vc in caches:
                    self.check(self.lib.mote_cuda_gqa_attention_decode_f16(
                        q.data_ptr(), kc.data_ptr(), vc.data_ptr(), lens.data_ptr(),
                        o.data_ptr(), batch, qh, kvh, hd, length, length, scale, ws.data_ptr(),
                        ws.numel(), self.stream()), "decode attention")
            g = self.graph(run)
            t = self.time_graph(g, 20, r) / r
            del g, caches
            out[f"decode_b{batch}_len{length}"] = {
                "us": round(t * 1e3, 2), "gbs": round(kv_bytes / t / 1e6, 1), "copies": r}
        for tokens in (512, 2048):
            kc = self.randn((tokens, kvh, hd), 7, torch.float16)
            vc = self.randn((tokens, kvh, hd), 8, torch.float16)
            q = self.randn((tokens, qh, hd), 9, torch.float16)
            o = torch.empty_like(q)

            def runp(kc=kc, vc=vc, q=q, o=o, tokens=tokens):
                self.check(self.lib.mote_cuda_gqa_attention_prefill_f16(
                    q.data_ptr(), kc.data_ptr(), vc.data_ptr(), o.data_ptr(), tokens, 0, qh,
                    kvh, hd, 0, tokens, scale, self.stream()), "prefill attention")
            g = self.graph(runp)
            t = self.time_graph(g, 20, 1)
            del g
            flops = 4.0 * hd * qh * tokens * (tokens + 1) / 2
            out[f"prefill_t{tokens}"] = {"us": round(t * 1e3, 2),
                                         "tflops": round(flops / t / 1e9, 1)}
        return out

    def sharded_linear(self, n: int, ms_list, seed: int, k: int = 4096) -> dict:
        """A linear column-sharded over the ranks (strong scaling): per step
        each rank runs the Q4_0 linear on its rows [rank * shard, ...) and the
        f16 outputs are all-gathered -- with NCCL (mote_cuda_comm_*), with the
        peer-store kernel, and fused into the GEMV or tcgen05 GEMM epilogue
        (stores into every rank's [M, N] output over NVLink + flag
        handshake).  Steps are captured in CUDA graphs; times are the max over
        ranks; GB/s counts the full weight once per step, TFLOP/s 2 M N K.  A
        shard smaller than 2.5x L2 is rotated over copies, one per step."""
        torch = self.torch
        import torch.distributed as dist

        from mote_b200 import comm

        sh = comm.shard_rows(n, self.world, self.rank)
        w0 = self.encode_q4_0(sh.rows, k, seed=seed + self.rank)
        ws = [w0] + [w0.clone() for _ in range(copies_for(w0.numel()) - 1)]
        fn = self.lib.mote_cuda_quantized_linear_q4_0_f16

        def exchange(obj):
            out = [None] * self.world
            dist.all_gather_object(out, obj)
            return out

        nccl = comm.NcclAllGather(self.world, self.rank, exchange)
        result = {"n": n, "k": k, "shard_rows": sh.rows, "world": self.world,
                  "weight_copies": len(ws)}
        steps = max(8, len(ws))
        try:
            for m in ms_list:
                reps = 10 if m <= 64 else 3
                x = self.randn((m, k), 60 + m, torch.float16)
                y = torch.empty((m, sh.rows), dtype=torch.float16, device=self.dev)
                count = m * sh.rows
                recv = torch.empty(self.world * count, dtype=torch.float16, device=self.dev)
                peer = comm.PeerAllGather(self.world, self.rank, count, exchange)
                fused = comm.ShardedLinearQ4_0(self.world, self.rank, m, n, k, exchange)

                def linear(i, x=x, y=y, m=m):
                    self.check(fn(x.data_ptr(), ws[i % len(ws)].data_ptr(), y.data_ptr(), m,
                                  sh.rows, k, self.stream()), "linear shard")

                def run_gemv():
                    for i in range(steps):
                        linear(i)

                def run_nccl(y=y, recv=recv, count=count):
                    for i in range(steps):
                        linear(i)
                        nccl.all_gather(y.data_ptr(), recv.data_ptr(), count, self.stream())

                def run_p2p(y=y, peer=peer):
                    for i in range(steps):
                        linear(i)
                        peer.all_gather(y.data_ptr(), i % 2, self.stream())

                def run_fused(x=x, fused=fused):
                    for i in range(steps):
                        fused(x.data_ptr(), ws[i % len(ws)].data_ptr(), i % 2, self.stream())

                row = {}
                # fused: the GEMV (<= 16 tokens) or the tcgen05 GEMM with the
                # peer-store epilogue and the handshake, one kernel per step
                arms = [("gemv", run_gemv, 1), ("nccl", run_nccl, 1), ("p2p", run_p2p, 2),
                        ("fused", run_fused, 1)]
                for name, body, kernels in arms:
                    self.barrier()
                    g = self.graph(body)
                    self.barrier()
                    t = self.max_over_ranks(self.time_graph(g, reps, steps * kernels)) / steps
                    del g
                    row[f"{name}_us"] = round(t * 1e3, 2)
                    if m > 64:
                        row[f"{name}_tflops"] = round(2.0 * m * n * k / t / 1e9, 1)
                    else:
                        row[f"{name}_gbs"] = round(linear_bytes(m, n, k) / t / 1e6, 1)
                row["parity"] = self.sharded_parity(
                    m, n, k, sh, seed, x, y, recv, count, ws, peer, fused, nccl, linear)
                result[f"m{m}"] = row
                self.barrier()
                peer.close(barrier=self.barrier)
                fused.close(barrier=self.barrier)
                del recv, y
        finally:
            torch.cuda.synchronize()
            nccl.close()
        return result

    def sharded_parity(self, m, n, k, sh, seed, x, y, recv, count, ws, peer, fused, nccl,
                       linear) -> dict:
        """After the timed arms: one more step of each transport, outside any
        graph, and checks of what the ranks hold.
        * On every rank the gathered [M, N] of the NCCL, peer-store and fused
          arms are equal bit for bit.
        * On rank 0 every rank's columns equal a single-GPU run of that
          rank's weight rows (regenerated from their seed) through the
          plain entry, bit for bit -- the same kernels, so the gather must
          move them unchanged.
        * On rank 0, 256 sampled columns are within 1e-3 normwise of a
          float64 accumulation of their decoded weights.
        * Every rank's device status word (bounded waits) is 0."""
        import numpy as np
        import torch.distributed as dist

        from mote_b200 import comm

        torch = self.torch
        linear(0)
        nccl.all_gather(y.data_ptr(), recv.data_ptr(), count, self.stream())
        via_nccl = comm.gathered_to_rows(recv.view(-1), m, sh).clone()
        ptr = peer.all_gather(y.data_ptr(), 0, self.stream())
        via_p2p = comm.gathered_to_rows(
            self.torch_view(ptr, self.world * count * 2).view(torch.float16), m, sh).clone()
        out = fused(x.data_ptr(), ws[0].data_ptr(), 0, self.stream())
        via_fused = self.torch_view(out, m * n * 2).view(torch.float16).view(m, n).clone()
        self.barrier()
        bits = lambda t: t.view(torch.int16)  # noqa: E731
        same = bool(torch.equal(bits(via_nccl), bits(via_p2p)) and
                    torch.equal(bits(via_nccl), bits(via_fused)))
        single_gpu = True
        f64_err = None
        if self.rank == 0:
            fn = self.lib.mote_cuda_quantized_linear_q4_0_f16
            cols = np.random.default_rng(seed).choice(n, min(256, n), replace=False)
            pitch = k // 32 * 18
            xs = x.float().cpu().numpy().astype(np.float64)
            want = np.empty((m, cols.size), np.float64)
            for r in range(self.world):
                part = comm.shard_rows(n, self.world, r)
                if part.real_rows == 0:
                    continue
                wr = self.encode_q4_0(part.rows, k, seed=seed + r)
                yr = torch.empty((m, part.rows), dtype=torch.float16, device=self.dev)
                self.check(fn(x.data_ptr(), wr.data_ptr(), yr.data_ptr(), m, part.rows, k,
                              self.stream()), "single-GPU shard")
                got = via_fused[:, part.start:part.stop]
                single_gpu &= bool(torch.equal(bits(yr[:, :part.real_rows]), bits(got)))
                mine = np.nonzero((cols >= part.start) & (cols < part.stop))[0]
                if mine.size:
                    raw = wr.cpu().numpy().reshape(part.rows, pitch)[cols[mine] - part.start]
                    want[:, mine] = xs @ dequant_q4_0_f64(raw, k).T
                del wr, yr
            got = via_fused[:, torch.as_tensor(cols, device=self.dev)].float().cpu().numpy()
            f64_err = float(np.max(np.abs(got - want)) / max(np.max(np.abs(want)), 1e-30))
        status = ctypes.c_uint(0)
        self.check(self.lib.mote_cuda_device_status(ctypes.byref(status), 1), "device status")
        flags = torch.tensor([int(same), int(single_gpu), int(status.value)],
                             device=self.dev, dtype=torch.int64)
        every = [torch.zeros_like(flags) for _ in range(self.world)]
        dist.all_gather(every, flags)
        every = [t.tolist() for t in every]
        ok = (all(e[0] == 1 and e[1] == 1 and e[2] == 0 for e in every) and
              (f64_err is None or f64_err <= 1e-3))
        return {"ok": ok, "transports_equal": [bool(e[0]) for e in every],
                "single_gpu_equal": bool(single_gpu) if self.rank == 0 else None,
                "normwise_vs_f64": None if f64_err is None else round(f64_err, 7),
                "device_status": [e[2] for e in every]}

    def norm_rope_row_split(self) -> dict:
        """Config 2 at N > 1: the T = 512 tokens split by rows, T/G per rank,
        no exchange (the tokens are independent); us per layer = max over
        ranks, inputs rotated over copies holding >= 2.5x L2 per rank."""
        torch = self.torch
        t_all, hidden, qh, kh, hd = 512, 2048, 32, 8, 64
        t = -(-t_all // self.world)
        nbytes = (2 * t * hidden + 2 * t * qh * hd + 2 * t * kh * hd) * 2 + hidden * 2 + \
            2 * t * (hd // 2) * 4
        r = copies_for(nbytes)
        pos = torch.arange(self.rank * t, self.rank * t + t, dtype=torch.int32, device=self.dev)
        cos = torch.empty((t, hd // 2), dtype=torch.float32, device=self.dev)
        sin = torch.empty_like(cos)
        self.check(self.lib.mote_cuda_rope_cos_sin_f32(pos.data_ptr(), cos.data_ptr(),
                                                       sin.data_ptr(), t, hd,
                                                       ctypes.c_double(10000.0), self.stream()),
                   "rope table")
        gamma = self.randn((hidden,), 3, torch.float16, 0.1, 1.0)
        sets = []
        for i in range(r):
            x = self.randn((t, hidden), 10 + i, torch.float16)
            q = self.randn((t, qh, hd), 1000 + i, torch.float16)
            kk = self.randn((t, kh, hd), 2000 + i, torch.float16)
            sets.append((x, torch.empty_like(x), q, torch.empty_like(q), kk, torch.empty_like(kk),
                         cos.clone(), sin.clone()))
        fn = self.lib.mote_cuda_rms_norm_rope_f16

        def run():
            for (x, xo, q, qo, kk, ko, c, s) in sets:
                self.check(fn(x.data_ptr(), gamma.data_ptr(), xo.data_ptr(), q.data_ptr(),
                              qo.data_ptr(), kk.data_ptr(), ko.data_ptr(), c.data_ptr(),
                              s.data_ptr(), t, hidden, qh, kh, hd, 0, ctypes.c_float(1e-6),
                              self.stream()), "norm+rope")

        self.barrier()
        g = self.graph(run)
        self.barrier()
        ms = self.max_over_ranks(self.time_graph(g, 20, r)) / r
        del g, sets
        return {"tokens_per_rank": t, "us_per_layer": round(ms * 1e3, 3),
                "gbs_total": round(nbytes * self.world / ms / 1e6, 1), "copies": r}

    # -- main -------------------------------------------------------------------
    def run(self) -> dict | None:
        torch = self.torch
        args = self.args
        peaks = measured_peaks()
        self.build_sweep()
        g = self.graph(self.sweep_step)
        for _ in range(args.warmup):
            g.replay()
        self.barrier()
        sampler = ClockSampler(self.local_rank) if self.rank == 0 else None
        if sampler:
            sampler.start()
            time.sleep(0.3)
        self.barrier()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            g.replay()
        end.record()
        end.synchronize()
        self.barrier()
        clocks = sampler.stop() if sampler else None
        ms = self.max_over_ranks(start.elapsed_time(end))
        self.launches += args.steps * self.sweep_launches
        timed_launches = args.steps * self.sweep_launches
        value = self.sweep_bytes * args.steps * self.world / (ms / 1e3) / 1e9

        # dominant kernel: per-case launch durations (graphs of one case each)
        cases = []
        kern_bytes = 0
        kern_ms = 0.0
        for m in SWEEP_M:
            for n in SWEEP_N:
                gc = self.graph(lambda m=m, n=n: self.sweep_case(m, n))
                r = len(self.sweep_w[n])
                per = self.time_graph(gc, 10, r) / r
                b = linear_bytes(m, n, SWEEP_K)
                kern_bytes += b
                kern_ms += per
                cases.append({"m": m, "n": n, "us": round(per * 1e3, 3),
                              "gbs": round(b / per / 1e6, 1)})
                del gc
        achieved = kern_bytes / kern_ms / 1e6
        result = None
        extra = {}
        if self.rank == 0:
            extra["config1_f32_m1_k2048_n2048"] = self.config1()
            extra["config2_rmsnorm_rope_t512"] = self.config2()
            extra["config4_decoder_layer_m1"] = self.config4()
            extra["config5"] = self.config5()
            extra["q8_0_linear"] = self.q8_0()
            extra["kquant_linear"] = self.kquant()
            extra["dense_matmul_f16_f32"] = self.dense_matmul()
            extra["gqa_attention"] = self.attention()
        e2e = self.e2e(max(3, min(args.steps, 20)))
        if self.world > 1:
            # the splits the data plane supports: lm_head and FFN up/gate by
            # output columns (decode GEMV), the prefill GEMM by output columns
            # (tcgen05), config 2 by token rows
            extra["lm_head_sharded"] = self.sharded_linear(128256, (1, 16, 64), seed=700)
            extra["ffn_up_sharded"] = self.sharded_linear(14336, (1, 16), seed=800)
            extra["prefill_sharded"] = self.sharded_linear(14336, (2048,), seed=900)
            extra["norm_rope_row_split"] = self.norm_rope_row_split()
        if self.rank == 0:
            cpu = cpu_baseline(budget_s=args.cpu_seconds)
            c2 = extra["config2_rmsnorm_rope_t512"]
            result = {
                "metric": METRIC, "value": round(value, 2), "unit": "GB/s",
                "n_gpus": self.world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f16",
                "data": "synthetic (seeded N(0,0.02) weights Q4_0-encoded on device, "
                        "N(0,1) f16 activations)",
                "config": sweep_config(self.world),
                "roofline": {
                    "bound": "hbm", "achieved": round(achieved, 1),
                    "peak": peaks["hbm_gbs"], "unit": "GB/s",
                    "frac": round(achieved / peaks["hbm_gbs"], 4),
                    "frac_of_8tbs_spec": round(achieved / SPEC_HBM_GBS, 4),
                    "peak_source": peaks["source"],
                    "traffic": (round(traffic_ratio() * kern_bytes / len(cases))
                                if traffic_ratio() else None),
                    "traffic_note": "ncu DRAM bytes / algorithmic bytes of the GEMV (lm_head "
                                    "capture, profiles/q4_0_gemv_lm_head_m1.txt) x the average "
                                    "algorithmic bytes of one sweep launch",
                    "kernel": "q4_0_gemv_kernel (average over the sweep cases below)"},
                "norm_rope_us_per_layer": c2["us_per_layer"],
                "norm_rope_roofline": {"bound": "hbm", "achieved": c2["gbs"],
                                       "peak": peaks["hbm_gbs"], "unit": "GB/s",
                                       "frac": round(c2["gbs"] / peaks["hbm_gbs"], 4)},
                "cpu_baseline": cpu,
                "e2e": e2e,
                "clocks": clocks,
                "gpu_launches": timed_launches,
                "cases": cases,
                "extra": extra,
            }
            if self.world > 1:
                rows = [(leg, key, r["parity"]) for leg in ("lm_head_sharded", "ffn_up_sharded",
                                                          "prefill_sharded")
                        for key, r in extra[leg].items() if isinstance(r, dict) and "parity" in r]
                result["sharded_parity"] = {
                    "ok": all(p_["ok"] for _, _, p_ in rows),
                    "device_status": sorted({st for _, _, p_ in rows
                                             for st in p_["device_status"]}),
                    "cases": {f"{leg}.{key}": p_["ok"] for leg, key, p_ in rows}}
                lm1 = extra["lm_head_sharded"]["m1"]
                result["lm_head_sharded_m1"] = {
                    "n_gpus": self.world, "fused_us": lm1["fused_us"], "p2p_us": lm1["p2p_us"],
                    "nccl_us": lm1["nccl_us"], "shard_gemv_us": lm1["gemv_us"],
                    "single_gpu_us": extra["config5"]["lm_head_m1"]["us"],
                    "note": "column-sharded lm_head K=4096 N=128256 M=1 (strong scaling): "
                            "max-over-ranks us per step"}
        if self.world > 1:
            self.barrier()
            self.torch.distributed.destroy_process_group()
        return result


def traffic_ratio():
    """(DRAM read + write) / algorithmic bytes of the GEMV, from the committed
    ncu summary (``traffic_ratio:`` line), or None."""
    path = ROOT / "profiles" / "q4_0_gemv_lm_head_m1.txt"
    try:
        for line in path.read_text().splitlines():
            if line.strip().startswith("traffic_ratio:"):
                return float(line.split(":", 1)[1].split()[0])
    except (OSError, ValueError, IndexError):
        return None
    return None


# --------------------------------------------------------------------------
CPU_SAMPLE_ROWS = 512


def dequant_q4_0_f64(rows, k: int):
    """Decoded Q4_0 rows [r, K/32*18] bytes -> float64 [r, K] (the block
    layout of crates/mote-reference/src/quantized.rs:177-201)."""
    import numpy as np

    b = np.asarray(rows, np.uint8).reshape(-1, k // 32, 18)
    d = b[:, :, 0:2].copy().view(np.float16).astype(np.float64)
    qs = b[:, :, 2:]
    q = np.concatenate([(qs & 15).astype(np.int16) - 8, (qs >> 4).astype(np.int16) - 8], axis=2)
    return (q * d).reshape(-1, k)


def sweep_config(world: int) -> dict:
    """The `config` of the headline line, shared by both arms."""
    return {
        "workload": "config3 batch-decode sweep: Q4_0 linear M in {1,2,4,8,16} x "
                    "N in {4096,11008,14336}, K=4096, f16 act, f32 acc, f16 out "
                    "(mote_cuda_quantized_linear_q4_0_f16_ws, one workspace)",
        "weight_copies_per_n": {str(n): copies_for(q4_bytes(n, SWEEP_K)) for n in SWEEP_N},
        "l2": "inputs larger than L2: each case rotates over copies holding "
              ">= 2.5x L2 (126 MB)",
        "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
        "timing": "CUDA graph per step, CUDA events, max over ranks"}


def cpu_sample(k: int = SWEEP_K, rows: int = CPU_SAMPLE_ROWS):
    """A bounded slice of the config-3 sweep for the CPU oracle: the first
    `rows` output features of each of the three N's matrices (seeded
    N(0, 0.02) weights, Q4_0-encoded) and the f16-valued activations of
    every M of the sweep.  The slice has every case of the sweep, each with
    the same number of rows, so per-row work (a K=4096 decode and M dot
    products) is weighted as in the full sweep."""
    import numpy as np

    from oracle import ref

    rng = np.random.default_rng(4096)
    ws = {}
    for n in SWEEP_N:
        ws[n] = ref.q4_0_quantize(rng.normal(0, 0.02, (rows, k)).astype(np.float32), rows, k)
    xs = {m: rng.normal(0, 1, (m, k)).astype(np.float16).astype(np.float32) for m in SWEEP_M}
    return ws, xs


def cpu_sample_bytes(k: int = SWEEP_K, rows: int = CPU_SAMPLE_ROWS) -> int:
    """Algorithmic bytes of one pass over the sample (weights once per call,
    x and y), the headline's byte count restricted to the sampled rows."""
    return sum(linear_bytes(m, rows, k) for m in SWEEP_M for _ in SWEEP_N)


def cpu_pass(ws, xs, threads: int, k: int = SWEEP_K, rows: int = CPU_SAMPLE_ROWS) -> None:
    from oracle import ref

    for m in SWEEP_M:
        for n in SWEEP_N:
            ref.quantized_linear_f32(xs[m], ws[n], ref.Q4_0, m, rows, k, threads=threads)


def cpu_sample_text(rows: int, threads: int, passes: int | None = None) -> str:
    head = f"{passes} passes of " if passes is not None else "per step: "
    return (f"{head}the 15 config-3 cases (M in {{1,2,4,8,16}} x N in {{4096,11008,14336}}, "
            f"K=4096), each on the first {rows} output features of its N, through "
            f"quantized_linear_f32 (mote-reference crates/mote-reference/src/quantized.rs:89-144 "
            f"restated in C, oracle/), {threads} thread(s)")


def cpu_baseline(budget_s: float = 10.0, threads: int = 1) -> dict:
    """The reference's CPU path, single-threaded as mote-reference's
    quantized_linear_f32 is (crates/mote-reference/src/quantized.rs:127-142),
    timed on this host over a bounded sample of the sweep."""
    from oracle import ref

    ref.build()
    ws, xs = cpu_sample()
    per_pass = cpu_sample_bytes()
    cpu_pass(ws, xs, threads)  # warm-up
    passes = 0
    t0 = time.perf_counter()
    while True:
        cpu_pass(ws, xs, threads)
        passes += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": round(per_pass * passes / dt / 1e9, 4), "unit": "GB/s", "cores": threads,
            "kind": "port" if threads == 1 else "ours",
            "sample": cpu_sample_text(CPU_SAMPLE_ROWS, threads, passes)}


def run_reference(args) -> None:
    """Reference arm: mote-reference's CPU linear (restated in C in oracle/;
    the Rust crate cannot be built here), single-threaded as the reference
    is, on the same metric and config as our arm, each step one pass over a
    bounded sample of the sweep (every case, the first rows of each N)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import ref

    ref.build()
    threads = 1
    ws, xs = cpu_sample()
    per_step = cpu_sample_bytes()
    for _ in range(args.warmup):
        cpu_pass(ws, xs, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_pass(ws, xs, threads)
    dt = time.perf_counter() - t0
    value = per_step * args.steps / dt / 1e9
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3 / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": sweep_config(args.gpus),
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads,
                         "kind": "port", "sample": cpu_sample_text(CPU_SAMPLE_ROWS, threads)},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def run_single_case(args) -> None:
    """One kernel, a few plain launches (no graph): the command ncu profiles.

    --only gemv       Q4_0 linear f16 -> f16, [--m, --n, --k]
    --only q8_0       Q8_0 linear f16 -> f16, [--m, --n, --k]
    --only q4_k       Q4_K linear f16 -> f16, [--m, --n, --k]
    --only q6_k       Q6_K linear f16 -> f16, [--m, --n, --k]
    --only norm_rope  fused RMSNorm + RoPE at config-2 geometry
    """
    import torch

    b = Bench(args)
    torch = b.torch
    times = []
    if args.only == "gemv":
        m, n, k = args.m, args.n, args.k
        w = b.encode_q4_0(n, k, seed=1)
        x = b.randn((m, k), 2, torch.float16)
        y = torch.empty((m, n), dtype=torch.float16, device=b.dev)

        if args.ws:
            # the workspace entry mote_b200.ops uses (K split over CTAs for
            # 9-16 tokens, split last wave on the tensor-core path)
            wsp = torch.zeros(max(b.workspace_bytes(m, n, k), 256), dtype=torch.uint8,
                              device=b.dev)

            def launch():
                b.check(b.lib.mote_cuda_quantized_linear_q4_0_f16_ws(
                    x.data_ptr(), w.data_ptr(), y.data_ptr(), m, n, k, wsp.data_ptr(),
                    wsp.numel(), b.stream()), "gemv")
        else:
            def launch():
                b.check(b.lib.mote_cuda_quantized_linear_q4_0_f16(
                    x.data_ptr(), w.data_ptr(), y.data_ptr(), m, n, k, b.stream()), "gemv")
        nbytes = linear_bytes(m, n, k)
    elif args.only == "q8_0":
        m, n, k = args.m, args.n, args.k
        nb = n * (k // 32) * 34
        g0 = torch.Generator(device=b.dev).manual_seed(1)
        w = torch.randint(0, 256, (nb,), generator=g0, dtype=torch.uint8, device=b.dev)
        blocks = w.view(n * (k // 32), 34)
        blocks[:, 0] = 0
        blocks[:, 1] = 0x20  # f16 scale bits 0x2000
        x = b.randn((m, k), 2, torch.float16)
        y = torch.empty((m, n), dtype=torch.float16, device=b.dev)

        def launch():
            b.check(b.lib.mote_cuda_quantized_linear_q8_0_f16(
                x.data_ptr(), w.data_ptr(), y.data_ptr(), m, n, k, b.stream()), "q8_0")
        nbytes = nb + m * k * 2 + m * n * 2
    elif args.only in ("q4_k", "q6_k"):
        m, n, k = args.m, args.n, args.k
        w, nb = b.kquant_weights(args.only, n, k, seed=1)
        x = b.randn((m, k), 2, torch.float16)
        y = torch.empty((m, n), dtype=torch.float16, device=b.dev)
        fn = getattr(b.lib, f"mote_cuda_quantized_linear_{args.only}_f16")

        def launch():
            b.check(fn(x.data_ptr(), w.data_ptr(), y.data_ptr(), m, n, k, b.stream()), args.only)
        nbytes = nb + m * k * 2 + m * n * 2
    elif args.only in ("attn_decode", "attn_prefill"):
        qh, kvh, hd = 32, 8, 64
        length = args.n if args.n != 128256 else 4096
        scale = ctypes.c_float(1.0 / math.sqrt(hd))
        if args.only == "attn_decode":
            batch = args.m
            kc = b.randn((batch * length, kvh, hd), 1, torch.float16)
            vc = b.randn((batch * length, kvh, hd), 2, torch.float16)
            q = b.randn((batch, qh, hd), 3, torch.float16)
            o = torch.empty_like(q)
            lens = torch.full((batch,), length, dtype=torch.int32, device=b.dev)
            need = ctypes.c_uint64(0)
            b.check(b.lib.mote_cuda_gqa_attention_decode_workspace_bytes(
                batch, qh, kvh, hd, length, ctypes.byref(need)), "workspace")
            ws = torch.empty(max(need.value, 16), dtype=torch.uint8, device=b.dev)

            def launch():
                b.check(b.lib.mote_cuda_gqa_attention_decode_f16(
                    q.data_ptr(), kc.data_ptr(), vc.data_ptr(), lens.data_ptr(), o.data_ptr(),
                    batch, qh, kvh, hd, length, length, scale, ws.data_ptr(), ws.numel(),
                    b.stream()), "decode attention")
            nbytes = 2 * batch * length * kvh * hd * 2
        else:
            kc = b.randn((length, kvh, hd), 1, torch.float16)
            vc = b.randn((length, kvh, hd), 2, torch.float16)
            q = b.randn((length, qh, hd), 3, torch.float16)
            o = torch.empty_like(q)

            def launch():
                b.check(b.lib.mote_cuda_gqa_attention_prefill_f16(
                    q.data_ptr(), kc.data_ptr(), vc.data_ptr(), o.data_ptr(), length, 0, qh, kvh,
                    hd, 0, length, scale, b.stream()), "prefill attention")
            nbytes = (3 * length * kvh * hd + 2 * length * qh * hd) * 2
    elif args.only == "norm_rope":
        t, hidden, qh, kh, hd = 512, 2048, 32, 8, 64
        pos = torch.arange(t, dtype=torch.int32, device=b.dev)
        cos = torch.empty((t, hd // 2), dtype=torch.float32, device=b.dev)
        sin = torch.empty_like(cos)
        b.check(b.lib.mote_cuda_rope_cos_sin_f32(pos.data_ptr(), cos.data_ptr(), sin.data_ptr(),
                                                 t, hd, ctypes.c_double(10000.0), b.stream()),
                "table")
        xs = b.randn((t, hidden), 1, torch.float16)
        gamma = b.randn((hidden,), 3, torch.float16, 0.1, 1.0)
        q = b.randn((t, qh, hd), 4, torch.float16)
        kk = b.randn((t, kh, hd), 5, torch.float16)
        xo, qo, ko = torch.empty_like(xs), torch.empty_like(q), torch.empty_like(kk)

        def launch():
            b.check(b.lib.mote_cuda_rms_norm_rope_f16(
                xs.data_ptr(), gamma.data_ptr(), xo.data_ptr(), q.data_ptr(), qo.data_ptr(),
                kk.data_ptr(), ko.data_ptr(), cos.data_ptr(), sin.data_ptr(), t, hidden, qh, kh,
                hd, 0, ctypes.c_float(1e-6), b.stream()), "norm_rope")
        nbytes = (2 * t * hidden + 2 * t * qh * hd + 2 * t * kh * hd) * 2 + hidden * 2 + \
            2 * t * (hd // 2) * 4
    elif args.only == "stack":
        # the persistent decoder stack: --m layers of Llama-3.2-1B shapes at one
        # token (distinct random weights; 4 layers = 137 MB > L2)
        import numpy as np

        from mote_b200 import decoder
        from mote_b200.context import CudaContext
        from mote_b200.types import DType, plain

        ctx = CudaContext(b.local_rank)
        shape = decoder.LayerShape()
        count = max(1, args.m)
        layers = [decoder.random_layer(ctx, shape, seed=70 + i, vocab=1000) for i in range(count)]
        rng = np.random.default_rng(0)
        for layer in layers:
            ctx.upload_numpy(layer.attn, rng.normal(0, 1, (1, shape.hidden)).astype(np.float16))
            layer.set_position(7)
        h_in = ctx.from_bytes(plain((1, shape.hidden), DType.F16),
                              rng.normal(0, 0.5, shape.hidden).astype(np.float16))
        st = decoder.DecoderStackQ4_0(ctx, layers)
        ctx.sync()
        torch.cuda.set_stream(torch.cuda.ExternalStream(ctx.stream))  # the events' stream

        def launch():
            st.run(h_in)
        nbytes = count * shape.weight_bytes()
    else:
        raise SystemExit(f"unknown --only {args.only}")
    for _ in range(args.launches):
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        launch()
        end.record()
        end.synchronize()
        times.append(start.elapsed_time(end))
    best = min(times)
    print(json.dumps({"only": args.only, "launches": args.launches, "best_us": round(best * 1e3, 2),
                      "gbs_at_best": round(nbytes / best / 1e6, 1), "bytes": nbytes}), flush=True)


def main() -> int:
    p = argparse.ArgumentParser()
    p.add_argument("--only", default=None,
                   help="profile one kernel: gemv | q8_0 | q4_k | q6_k | norm_rope | "
                        "attn_decode (--m batch, --n length) | attn_prefill (--n tokens) | "
                        "stack (--m layers)")
    p.add_argument("--m", type=int, default=1)
    p.add_argument("--n", type=int, default=128256)
    p.add_argument("--k", type=int, default=4096)
    p.add_argument("--launches", type=int, default=3)
    p.add_argument("--ws", action="store_true",
                   help="--only gemv: the workspace entry (as mote_b200.ops calls it)")
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--cpu-seconds", type=float, default=10.0)
    args = p.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
        return 0
    if args.only:
        run_single_case(args)
        return 0
    from mote_b200 import build as _b

    if not _b.LIB_PATH.exists():
        raise SystemExit("libmote_cuda.so missing: run python -m mote_b200.build")
    # Libraries (NCCL's version banner, for one) may write to file
    # descriptor 1; keep it for the one JSON line and send the rest to stderr.
    sys.stdout.flush()
    json_fd = os.dup(1)
    os.dup2(2, 1)
    try:
        result = Bench(args).run()
    finally:
        sys.stdout.flush()
        os.dup2(json_fd, 1)
        os.close(json_fd)
    if result is not None:
        print(json.dumps(result), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
