"""Benchmark of the B200 attention hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl ours|reference]

Configurations (BASELINE.json "configs", synthetic seeded data):
  prefill  causal prefill SDPA, S 4096, Hq 16 / Hkv 4 / d 256, gated     TFLOP/s
  decode   one decode step, n 2048, same heads, gated                    GB/s
  gdn      GatedDeltaNet: prefill T 4096 then 256 decode steps           tok/s
  batch    batched decode, 64 sequences, L ~ U{1024..32768}              GB/s
  cp       causal prefill SDPA at S 131072, context parallel over the GPUs
           (zig-zag shards, K/V ring by NCCL send/recv, LSE merge)      TFLOP/s  (default)
           one GPU runs the whole sequence through the single-GPU kernel
  cp_hops  the ring's hop kernel alone: rank 3 of an 8-rank ring emulated on
           one GPU (all shards resident, no transport), hops + finish   TFLOP/s
  front    attention front end of a 4096-row block: q/k head norms,
           partial RoPE, KV append                                      GB/s
  gdn_front  DeltaNet front end of a 4096-row block: causal conv + SiLU
           over qkv (8192 channels, K 4), beta/decay gates               GB/s
  gdn_norm   DeltaNet gated RMS norm of a 4096-row block (32 V heads)    GB/s
  mixers     one decode token through the mixers of all 32 layers of a hybrid
           model (8 attention at 32768 positions, 24 DeltaNet) routed by an
           hb_mount: per layer the front end, attention or recurrence, and
           the gated norm; the projections are not part of it             tok/s
  snapshot   snapshot of a hybrid model's state at 32768 positions into a
           pinned host image in the reference's format (8 attention layers'
           KV, 24 DeltaNet layers' states, logits); e2e adds the restore  GB/s
A step is one pass of the path over one batch: one prefill / one decode step /
one GDN prefill + 256 steps / one decode step of the whole batch / one
131072-token prefill / one front-end (or gated-norm) call.  The ring holds
NCCL calls, so `cp` steps are issued eagerly between the CUDA events instead
of from a CUDA graph (a step lasts tens of milliseconds; launch costs are
microseconds).

`--gpus N` without torchrun starts N ranks with torch.distributed.run;
under torchrun N must equal WORLD_SIZE.

`value` is device-timed with CUDA events on the launching stream around one
CUDA-graph replay of K steps, inputs resident in HBM and rotated over copies
whose total exceeds twice the 126 MB L2 (so every step reads cold inputs);
under torchrun the timed total is the max over ranks.  `e2e` is the same metric
through the C ABI with inputs copied from pinned host memory and the result
copied back inside the timed region.  `--impl reference` times the CPU
restatement of the reference's x86 kernels (the oracle) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.join(ROOT, "herbert-jit-bf16_b200")]

HQ, HKV, HD = 16, 4, 256
NK, NV, HKD, HVD = 16, 32, 128, 128
PREFILL_S = 4096
# cached positions of the decode configuration (BASELINE configs[0] at
# 2048); HB_DECODE_N measures the same step over a longer cache
DECODE_N = int(os.environ.get("HB_DECODE_N", 2048))
GDN_T, GDN_STEPS = 4096, 256
CP_S = 131072
FRONT_ROTARY = 64  # Qwen3.5: partial_rotary_factor 0.25 of head_dim 256
L2_BYTES = 126 << 20

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of
# each configuration's dominant kernel, as an ncu capture of this script's
# own command measured them.  ncu runs outside the timed run (a capture
# replays kernels and is never timed), so the figures are constants here;
# batch is scaled from the n = 2048 decode capture by the bytes processed,
# gdn covers the chunked prefill's kernels of one prefill, cp is the
# single-GPU prefill of the whole sequence (the ring's hops are other
# launches), and None marks a configuration whose launch was not captured.
NCU_TRAFFIC = {"prefill": 93_118_464, "decode": 8_439_296, "gdn": 504_317_696,
               "batch": 4_633_303_808, "cp": 39_260_000_000, "cp_hops": None, "front": 56_784_128,
               "gdn_front": 213_700_000, "gdn_norm": 153_000_000, "snapshot": None,
               "mixers": None}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            j = json.load(f)
        return {"hbm": float(j["hbm_gbs"]), "bf16": float(j["bf16_tflops"]),
                "bf16_sustained": float(j.get("bf16_tflops_sustained", j["bf16_tflops"])),
                "source": "measured"}
    except Exception:
        return {"hbm": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


def prefill_flops(S, past=0, heads=HQ, hd=HD):
    n = sum(range(past + 1, past + S + 1))
    return 4.0 * heads * hd * n


def gdn_prefill_flops(T, nv=NV, dk=HKD, dv=HVD, C=64):
    per = 6 * C * dk * dv + 6 * C * C * dk + 4 * C * C * dv + C ** 3 / 3
    return per * (T // C) * nv


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi samples of the SM clock and throttle reasons, every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def start(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits", "-i", str(self.idx)],
                                     capture_output=True, text=True, timeout=5).stdout
                for line in out.strip().splitlines():
                    self.samples.append([x.strip() for x in line.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def stop(self):
        self._stop.set()
        if self._t:
            self._t.join(timeout=10)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for s in self.samples:
            try:
                sm.append(float(s[1]))
                mx = float(s[2])
                for n, v in zip(names, s[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
            except Exception:
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def smi_index(dev):
    """nvidia-smi index of torch device `dev` (matched by PCI bus id)."""
    import torch
    try:
        bus = torch.cuda.get_device_properties(dev).pci_bus_id.lower()
        out = subprocess.run(["nvidia-smi", "--query-gpu=index,pci.bus_id",
                              "--format=csv,noheader"], capture_output=True, text=True,
                             timeout=10).stdout
        for line in out.strip().splitlines():
            i, b = [x.strip().lower() for x in line.split(",")]
            if b.endswith(bus[-12:]) or bus.endswith(b[-12:]):
                return int(i)
    except Exception:
        pass
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    ids = [x for x in vis.split(",") if x.strip().isdigit()]
    return int(ids[dev]) if dev < len(ids) else dev


# --------------------------------------------------------------- workloads

class Workload:
    """One configuration on one GPU.

    `sets` holds R copies of the step's inputs (R chosen so that the copies
    exceed twice the L2); step(i) runs the path on copy i % R with inputs
    resident in HBM; e2e_step(i) copies the step's inputs from pinned host
    memory, runs the path and copies the result back."""

    launches_per_step = 1
    graphable = True

    @staticmethod
    def rotation(bytes_per_set):
        return max(1, -(-2 * L2_BYTES // max(1, bytes_per_set)))


def _randn_bf16(shape, gen, device):
    import torch
    return torch.randn(shape, generator=gen, device=device, dtype=torch.float32).to(
        torch.bfloat16)


def _nbytes(*ts):
    return sum(t.numel() * t.element_size() for t in ts)


class _AttnWorkload(Workload):
    """Shared by the prefill and single-sequence decode configurations."""

    def __init__(self, device, rows, past, seed):
        import torch
        import herbert_b200 as hb
        self.hb, self.rows, self.past = hb, rows, past
        n = past + rows
        gen = torch.Generator(device=device).manual_seed(seed)
        qd = HQ * HD
        per_set = (rows * 2 * qd + 2 * HKV * n * HD + rows * qd) * 2
        self.R = self.rotation(per_set)
        self.sets = []
        for _ in range(self.R):
            self.sets.append((_randn_bf16((rows, 2 * qd), gen, device),
                              _randn_bf16((HKV, n, HD), gen, device),
                              _randn_bf16((HKV, n, HD), gen, device),
                              torch.empty((rows, qd), dtype=torch.bfloat16, device=device)))
        self.spec = hb.attention_spec(HQ, HQ // HKV, HD, True)
        self.ws = None
        q, k, v, out = self.sets[0]
        self.h_in = [t.cpu().pin_memory() for t in (q, k, v)]
        self.h_out = torch.empty(out.shape, dtype=out.dtype).pin_memory()
        self.h2d = _nbytes(*self.h_in)
        self.d2h = _nbytes(self.h_out)
        self.set_bytes = per_set

    def step(self, i=0):
        q, k, v, out = self.sets[i % self.R]
        n = self.past + self.rows
        self.ws = self.hb.attention(self.spec, q, k, v, out, rows=self.rows, past=self.past,
                                    kv_stride=n * HD, capacity=n, regime=self.regime,
                                    workspace=self.ws)

    def e2e_step(self, i=0):
        q, k, v, out = self.sets[0]
        n = self.past + self.rows
        if self.regime == "prefill":
            # hb_attn_prefill_host: the copies of each block of rows overlap
            # the computation of the others
            self.ws = self.hb.prefill_host(self.spec, *self.h_in, self.h_out, q, k, v, out,
                                           rows=self.rows, past=self.past, kv_stride=n * HD,
                                           capacity=n, workspace=self.ws)
            return
        for d, h in zip((q, k, v), self.h_in):
            d.copy_(h, non_blocking=True)
        self.step(0)
        self.h_out.copy_(out, non_blocking=True)


class PrefillWorkload(_AttnWorkload):
    regime = "prefill"

    def __init__(self, device, S=PREFILL_S, seed=0x5EED0002):
        super().__init__(device, S, 0, seed)
        self.S = S
        self.work = prefill_flops(S)
        self.units = "TFLOP/s"



class DecodeWorkload(_AttnWorkload):
    regime = "decode"

    def __init__(self, device, n=DECODE_N, seed=0x5EED0001):
        super().__init__(device, 1, n - 1, seed)
        self.n = n
        self.work = 2 * HKV * n * HD * 2 + 3 * HQ * HD * 2  # K+V + q + gate + out bytes
        self.units = "GB/s"



class GdnWorkload(Workload):
    def __init__(self, device, T=GDN_T, steps=GDN_STEPS, seed=0x5EED0003):
        import torch
        import herbert_b200 as hb
        self.hb, self.T, self.steps = hb, T, steps
        gen = torch.Generator(device=device).manual_seed(seed)
        conv = 2 * NK * HKD + NV * HVD
        rows = T + steps
        per_set = rows * (conv + 2 * NV + NV * HVD) * 4
        self.R = self.rotation(per_set)
        self.sets = []
        for _ in range(self.R):
            qkv = _randn_bf16((rows, conv), gen, device).float()
            b = torch.randn((rows, NV), generator=gen, device=device)
            g = torch.randn((rows, NV), generator=gen, device=device)
            self.sets.append((qkv, torch.sigmoid(b),
                              torch.exp(-torch.nn.functional.softplus(g)),
                              torch.empty((rows, NV * HVD), dtype=torch.float32, device=device)))
        self.state = torch.zeros((NV, HKD, HVD), dtype=torch.float32, device=device)
        self.shape = hb.DeltaShape(nk=NK, nv=NV, hkd=HKD, hvd=HVD)
        self.ws = None
        self.work = T + steps
        self.units = "tok/s"
        self.launches_per_step = 2 + steps  # prep + scan, then one kernel per decode step
        qkv, beta, decay, out = self.sets[0]
        self.h_in = [t.cpu().pin_memory() for t in (qkv, beta, decay)]
        self.h_out = torch.empty(out.shape, dtype=out.dtype).pin_memory()
        self.h2d = _nbytes(*self.h_in)
        self.d2h = _nbytes(self.h_out)
        self.set_bytes = per_set

    def step(self, i=0):
        hb = self.hb
        qkv, beta, decay, out = self.sets[i % self.R]
        self.state.zero_()
        self.ws = hb.delta_recurrence(self.shape, self.state, out, qkv, beta, decay,
                                      rows=self.T, regime="prefill", workspace=self.ws)
        for t in range(self.T, self.T + self.steps):
            hb.delta_recurrence(self.shape, self.state, out[t], qkv[t], beta[t], decay[t],
                                rows=1, regime="decode")

    def e2e_step(self, i=0):
        """The step from host buffers: the prefill rows through
        hb_gdn_prefill_host (each block's copies overlapped with the blocks
        before it), the decode rows' inputs copied on a side stream meanwhile,
        then the one-row steps and their outputs back."""
        import torch
        hb, T = self.hb, self.T
        qkv, beta, decay, out = self.sets[0]
        h_qkv, h_beta, h_decay = self.h_in
        cur = torch.cuda.current_stream()
        if not hasattr(self, "side"):
            self.side = torch.cuda.Stream()
        self.side.wait_stream(cur)
        with torch.cuda.stream(self.side):
            for d, h in zip((qkv, beta, decay), self.h_in):
                d[T:].copy_(h[T:], non_blocking=True)
        self.state.zero_()
        self.ws = hb.delta_prefill_host(self.shape, self.state, out, qkv, beta, decay, h_qkv,
                                        h_beta, h_decay, self.h_out, rows=T, workspace=self.ws)
        cur.wait_stream(self.side)
        for t in range(T, T + self.steps):
            hb.delta_recurrence(self.shape, self.state, out[t], qkv[t], beta[t], decay[t],
                                rows=1, regime="decode")
        self.h_out[T:].copy_(out[T:], non_blocking=True)

    def kernel_probe(self, reps=5):
        """(FLOPs, seconds) of one chunked prefill (prep + scan kernels), by
        CUDA events on the launching stream."""
        import torch
        qkv, beta, decay, out = self.sets[0]
        st = torch.cuda.current_stream()

        def fn():
            self.ws = self.hb.delta_recurrence(self.shape, self.state, out, qkv, beta, decay,
                                               rows=self.T, regime="prefill", workspace=self.ws)
        fn()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record(st)
        for _ in range(reps):
            fn()
        b.record(st)
        torch.cuda.synchronize()
        return gdn_prefill_flops(self.T), a.elapsed_time(b) / 1e3 / reps



class BatchWorkload(Workload):
    def __init__(self, device, rank=0, world=1, seed=0x5EED0004):
        import torch
        import herbert_b200 as hb
        from herbert_b200.inputs import batch_lengths
        self.hb = hb
        lens = batch_lengths(64, 1024, 32768, seed)
        # the new token is position L-1: the cache holds L keys; every rank
        # derives the same plan (longest first, least-loaded GPU)
        mine = hb.shard_of(lens, world, rank)
        self.lens = [int(lens[i]) for i in mine]
        gen = torch.Generator(device=device).manual_seed(seed + rank)
        qd = HQ * HD
        self.caches, seqs = [], []
        self.q = _randn_bf16((len(mine), 2 * qd), gen, device)
        self.out = torch.empty((len(mine), qd), dtype=torch.bfloat16, device=device)
        for j, L in enumerate(self.lens):
            kv = _randn_bf16((2, HKV, L, HD), gen, device)
            self.caches.append(kv)
            seqs.append(hb.DecodeSeq(q=self.q[j].data_ptr(), keys=kv[0].data_ptr(),
                                     values=kv[1].data_ptr(), output=self.out[j].data_ptr(),
                                     past=L - 1, kv_stride=L * HD))
        self.table = hb.seq_table(seqs, device)
        self.spec = hb.attention_spec(HQ, HQ // HKV, HD, True)
        self.ws = None
        self.work = sum(4 * HKV * L * HD for L in self.lens) + len(self.lens) * 3 * qd * 2
        self.units = "GB/s"
        self.R = 1
        self.set_bytes = self.work
        self.h_in = [self.q.cpu().pin_memory()]
        self.h_out = torch.empty(self.out.shape, dtype=self.out.dtype).pin_memory()
        self.h2d = _nbytes(*self.h_in)
        self.d2h = _nbytes(self.h_out)

    def step(self, i=0):
        self.ws = self.hb.decode_batch(self.spec, self.table, len(self.lens),
                                       max(self.lens) - 1, sum(self.lens) - len(self.lens),
                                       workspace=self.ws)

    def e2e_step(self, i=0):
        # a decode step of a serving loop: the new query rows arrive from the
        # host, the caches are already resident, the outputs go back
        self.q.copy_(self.h_in[0], non_blocking=True)
        self.step()
        self.h_out.copy_(self.out, non_blocking=True)



class CpWorkload(Workload):
    """Config 5: S = 131072 causal prefill, rank r holding the zig-zag shard of
    chunks r and 2P-1-r (q rows, K and V); one GPU runs the whole sequence
    through the single-GPU prefill kernel."""
    graphable = False

    def __init__(self, device, rank=0, world=1, seed=0x5EED0005):
        import torch
        import herbert_b200 as hb
        if CP_S % (2 * world * 128):
            raise SystemExit(f"cp: {CP_S} tokens do not split into 2x{world} chunks of 128-row tiles")
        self.hb, self.rank, self.world = hb, rank, world
        c = CP_S // (2 * world)
        self.chunk = c
        self.cp = hb.cp_spec(world, rank, c)
        gen = torch.Generator(device=device).manual_seed(seed + rank)
        qd = HQ * HD
        self.q = _randn_bf16((2 * c, 2 * qd), gen, device)
        self.kv = _randn_bf16((2, HKV, 2 * c, HD), gen, device)
        self.out = torch.empty((2 * c, qd), dtype=torch.bfloat16, device=device)
        self.spec = hb.attention_spec(HQ, HQ // HKV, HD, True)
        self.comm = hb.CpComm() if world > 1 else None
        self.side = torch.cuda.Stream(device=device, priority=-1) if world > 1 else None
        self.ws = None
        pos = hb.cp_positions(self.cp, rank)
        self.work = 4 * HQ * HD * sum(p + 1 for p in pos)
        self.units = "TFLOP/s"
        self.launches_per_step = world + 1 if world > 1 else 1  # hops + finish
        self.R = 1
        self.set_bytes = _nbytes(self.q, self.kv, self.out)
        self.h_in = [self.q.cpu().pin_memory(), self.kv.cpu().pin_memory()]
        self.h_out = torch.empty(self.out.shape, dtype=self.out.dtype).pin_memory()
        self.h2d = _nbytes(*self.h_in)
        self.d2h = _nbytes(self.h_out)

    def step(self, i=0):
        self.ws = self.hb.prefill_cp(self.spec, self.cp, self.q, self.kv[0], self.kv[1], self.out,
                                     kv_stride=2 * self.chunk * HD, capacity=2 * self.chunk,
                                     comm=self.comm, workspace=self.ws, comm_stream=self.side)

    def e2e_step(self, i=0):
        if self.world == 1:
            # hb_attn_prefill_host: the copies of each block of rows overlap
            # the computation of the others
            c = self.chunk
            self.ws = self.hb.prefill_host(self.spec, self.h_in[0], self.h_in[1][0], self.h_in[1][1],
                                           self.h_out, self.q, self.kv[0], self.kv[1], self.out,
                                           rows=2 * c, past=0, kv_stride=2 * c * HD,
                                           capacity=2 * c, workspace=self.ws)
            return
        self.q.copy_(self.h_in[0], non_blocking=True)
        self.kv.copy_(self.h_in[1], non_blocking=True)
        self.step()
        self.h_out.copy_(self.out, non_blocking=True)

    def kernel_probe(self, reps=3):
        """(algorithmic FLOPs, seconds) of one launch of the dominant kernel, by
        CUDA events on its stream: the whole-sequence prefill on one GPU, the
        hop over the rank's own shard (hop 0) on a ring."""
        import torch
        st = torch.cuda.current_stream()
        c = self.chunk
        if self.world == 1:
            fn, flops = self.step, self.work
        else:
            def fn():
                self.hb.prefill_cp_hop(self.spec, self.cp, self.q, self.kv[0], self.kv[1],
                                       self.out, 0, kv_stride=2 * c * HD, capacity=2 * c,
                                       workspace=self.ws)
            # chunk r vs r and 2P-1-r vs 2P-1-r (diagonals), 2P-1-r vs r (full)
            flops = 4 * HQ * HD * (c * (c + 1) + c * c)
        fn()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record(st)
        for _ in range(reps):
            fn()
        b.record(st)
        torch.cuda.synchronize()
        return flops, a.elapsed_time(b) / 1e3 / reps

    def close(self):
        if self.comm is not None:
            self.comm.close()



CP_HOPS_RANKS, CP_HOPS_RANK = 8, 3


def cp_hops_chunk():
    """Chunk of the emulated ring: CP_S / (2 x 8) unless HB_CP_HOPS_CHUNK sets
    a smaller case (for a full ncu capture of one hop)."""
    return int(os.environ.get("HB_CP_HOPS_CHUNK", CP_S // (2 * CP_HOPS_RANKS)))


class CpHopsWorkload(Workload):
    """The hop kernel of the context-parallel ring on one GPU: rank
    CP_HOPS_RANK of an emulated ring of CP_HOPS_RANKS over the 131072-token
    sequence, its hops through hb_attn_prefill_cp_hop over every rank's shard
    (all shards resident, the transport left out) and the finishing step.  A
    step is that rank's causal work; the hops of a real ring rank are these
    launches with NCCL transfers beside them."""

    def __init__(self, device, seed=0x5EED000B):
        import torch
        import herbert_b200 as hb
        P, r = CP_HOPS_RANKS, CP_HOPS_RANK
        c = cp_hops_chunk()
        self.hb, self.chunk = hb, c
        self.cp = hb.cp_spec(P, r, c)
        gen = torch.Generator(device=device).manual_seed(seed)
        qd = HQ * HD
        self.q = _randn_bf16((2 * c, 2 * qd), gen, device)
        self.shards = [_randn_bf16((2, HKV, 2 * c, HD), gen, device) for _ in range(P)]
        self.out = torch.empty((2 * c, qd), dtype=torch.bfloat16, device=device)
        self.spec = hb.attention_spec(HQ, HQ // HKV, HD, True)
        self.ws = None
        pos = hb.cp_positions(self.cp, r)
        self.work = 4 * HQ * HD * sum(p + 1 for p in pos)
        self.units = "TFLOP/s"
        self.launches_per_step = P + 1
        self.R = 1
        self.set_bytes = _nbytes(self.q, self.out, *self.shards)
        self.h_in = [self.q.cpu().pin_memory()]
        self.h_out = torch.empty(self.out.shape, dtype=self.out.dtype).pin_memory()
        self.h2d = _nbytes(*self.h_in)
        self.d2h = _nbytes(self.h_out)

    def step(self, i=0):
        kvs = 2 * self.chunk * HD
        for hop in range(CP_HOPS_RANKS):
            sh = self.shards[self.hb.cp_hop_source(self.cp, hop)]
            self.ws = self.hb.prefill_cp_hop(self.spec, self.cp, self.q, sh[0], sh[1], self.out,
                                             hop, kv_stride=kvs, workspace=self.ws)
        own = self.shards[CP_HOPS_RANK]
        self.hb.prefill_cp_finish(self.spec, self.cp, self.q, own[0], own[1], self.out,
                                  kv_stride=kvs, workspace=self.ws)

    def e2e_step(self, i=0):
        self.q.copy_(self.h_in[0], non_blocking=True)
        self.step()
        self.h_out.copy_(self.out, non_blocking=True)


def front_bytes(rows, heads=HQ, kv_heads=HKV, hd=HD, rotary=FRONT_ROTARY):
    """Algorithmic bytes of one front-end call: q heads read and written, k
    read and written (in place) and written to the cache, v read and written
    to the cache, the two table rows read."""
    return rows * (2 * heads * hd * 2 + 3 * kv_heads * hd * 2 + 2 * kv_heads * hd * 2
                   + 2 * (rotary // 2) * 2)


class FrontWorkload(Workload):
    """Head-norm-rope of q and k plus kv-append for one 4096-row block at
    Qwen3.5 geometry (the front end of the S = 4096 prefill)."""

    def __init__(self, device, rows=PREFILL_S, seed=0x5EED0006):
        import torch
        import herbert_b200 as hb
        self.hb, self.rows = hb, rows
        gen = torch.Generator(device=device).manual_seed(seed)
        qd, kvd = HQ * HD, HKV * HD
        per_set = (rows * 2 * qd + 2 * rows * kvd + 2 * HKV * rows * HD) * 2
        self.R = self.rotation(per_set)
        self.sets = []
        for _ in range(self.R):
            self.sets.append((_randn_bf16((rows, 2 * qd), gen, device),
                              _randn_bf16((rows, kvd), gen, device),
                              _randn_bf16((rows, kvd), gen, device),
                              torch.empty((HKV, rows, HD), dtype=torch.bfloat16, device=device),
                              torch.empty((HKV, rows, HD), dtype=torch.bfloat16, device=device)))
        self.q_norm = (0.1 * torch.randn(HD, generator=gen, device=device)).to(torch.bfloat16)
        self.k_norm = (0.1 * torch.randn(HD, generator=gen, device=device)).to(torch.bfloat16)
        half = FRONT_ROTARY // 2
        pos = torch.arange(rows, dtype=torch.float64, device=device)[:, None]
        inv = 1e7 ** (-torch.arange(half, dtype=torch.float64, device=device) * 2 / FRONT_ROTARY)
        self.cos = torch.cos(pos * inv).to(torch.bfloat16)
        self.sin = torch.sin(pos * inv).to(torch.bfloat16)
        self.spec = hb.attention_spec(HQ, HQ // HKV, HD, True)
        self.kv = hb.KvSpec(heads=HKV, head_dim=HD, stride=rows * HD, capacity=rows,
                            max_batch=rows)
        self.work = front_bytes(rows)
        self.units = "GB/s"
        q, k, v, _, _ = self.sets[0]
        self.h_in = [t.cpu().pin_memory() for t in (q, k, v)]
        self.h_out = torch.empty(q.shape, dtype=q.dtype).pin_memory()
        self.h2d = _nbytes(*self.h_in)
        self.d2h = _nbytes(self.h_out)
        self.set_bytes = per_set

    def step(self, i=0):
        q, k, v, keys, values = self.sets[i % self.R]
        self.hb.attn_front(self.spec, self.kv, q, k, v, self.q_norm, self.k_norm, self.cos,
                           self.sin, rows=self.rows, past=0, rotary=FRONT_ROTARY, eps=1e-6,
                           gemma=True, keys=keys, values=values)

    def e2e_step(self, i=0):
        q, k, v, _, _ = self.sets[0]
        for d, h in zip((q, k, v), self.h_in):
            d.copy_(h, non_blocking=True)
        self.step(0)
        self.h_out.copy_(q, non_blocking=True)



def gdn_front_bytes(rows, nk=NK, nv=NV, hkd=HKD, hvd=HVD, ck=4):
    """Algorithmic bytes of one DeltaNet front-end call: qkv read and written
    (in place), the conv state read and written, the conv weights, ab read,
    beta and decay written, dt_bias and a_log."""
    conv = 2 * nk * hkd + nv * hvd
    return (rows * conv * 4 * 2 + conv * ck * 4 * 2 + conv * ck * 2 + rows * 2 * nv * 4
            + rows * nv * 4 * 2 + nv * 2 + nv * 4)


def gdn_norm_bytes(rows, nv=NV, hvd=HVD):
    """Algorithmic bytes of one gated-norm call: x and z read (f32), the bf16
    output written, the weight read (the f32 copy is not written)."""
    return rows * nv * hvd * (4 + 4 + 2) + hvd * 2


class GdnFrontWorkload(Workload):
    """Causal conv + SiLU over the qkv projection (in place) and the beta /
    decay gates for one 4096-row block at Qwen3.5 geometry."""

    def __init__(self, device, rows=GDN_T, seed=0x5EED0007):
        import torch
        import herbert_b200 as hb
        self.hb, self.rows = hb, rows
        gen = torch.Generator(device=device).manual_seed(seed)
        conv = 2 * NK * HKD + NV * HVD
        self.shape = hb.DeltaShape(nk=NK, nv=NV, hkd=HKD, hvd=HVD)
        per_set = rows * conv * 4 + rows * 2 * NV * 4 + rows * NV * 4 * 2
        self.R = self.rotation(per_set)
        self.sets = []
        for _ in range(self.R):
            self.sets.append((torch.randn((rows, conv), generator=gen, device=device),
                              2.0 * torch.randn((rows, 2 * NV), generator=gen, device=device),
                              torch.empty((rows, NV), dtype=torch.float32, device=device),
                              torch.empty((rows, NV), dtype=torch.float32, device=device)))
        self.state = torch.randn((conv, 4), generator=gen, device=device)
        self.weight = (0.25 * torch.randn((conv, 4), generator=gen, device=device)).to(
            torch.bfloat16)
        dt = torch.exp(torch.empty(NV, device=device).uniform_(-6.9, -2.3, generator=gen))
        self.dt_bias = (dt + torch.log(-torch.expm1(-dt))).to(torch.bfloat16)
        self.a_log = torch.log(torch.empty(NV, device=device).uniform_(1.0, 16.0, generator=gen))
        self.ws = hb.Workspace(256, device)
        self.work = gdn_front_bytes(rows)
        self.units = "GB/s"
        qkv, ab, beta, decay = self.sets[0]
        self.h_in = [t.cpu().pin_memory() for t in (qkv, ab)]
        self.h_out = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in (qkv, beta, decay)]
        self.h2d = _nbytes(*self.h_in)
        self.d2h = _nbytes(*self.h_out)
        self.set_bytes = per_set

    def step(self, i=0):
        qkv, ab, beta, decay = self.sets[i % self.R]
        self.hb.delta_front(self.shape, qkv, self.state, self.weight, ab, self.dt_bias,
                            self.a_log, beta, decay, rows=self.rows, ck=4, workspace=self.ws)

    def e2e_step(self, i=0):
        qkv, ab, beta, decay = self.sets[0]
        for d, h in zip((qkv, ab), self.h_in):
            d.copy_(h, non_blocking=True)
        self.step(0)
        for h, d in zip(self.h_out, (qkv, beta, decay)):
            h.copy_(d, non_blocking=True)



class GdnNormWorkload(Workload):
    """Gated RMS norm of the recurrence output for one 4096-row block at
    Qwen3.5 geometry (bf16 output only, the out-projection's input)."""

    def __init__(self, device, rows=GDN_T, seed=0x5EED0008):
        import torch
        import herbert_b200 as hb
        self.hb, self.rows = hb, rows
        gen = torch.Generator(device=device).manual_seed(seed)
        self.shape = hb.DeltaShape(nk=NK, nv=NV, hkd=HKD, hvd=HVD)
        vd = NV * HVD
        per_set = rows * vd * (4 + 4 + 2)
        self.R = self.rotation(per_set)
        self.sets = []
        for _ in range(self.R):
            self.sets.append((0.05 * torch.randn((rows, vd), generator=gen, device=device),
                              torch.randn((rows, vd), generator=gen, device=device),
                              torch.empty((rows, vd), dtype=torch.bfloat16, device=device)))
        self.weight = (1.0 + 0.1 * torch.randn(HVD, generator=gen, device=device)).to(
            torch.bfloat16)
        self.work = gdn_norm_bytes(rows)
        self.units = "GB/s"
        x, z, out = self.sets[0]
        self.h_in = [t.cpu().pin_memory() for t in (x, z)]
        self.h_out = torch.empty(out.shape, dtype=out.dtype).pin_memory()
        self.h2d = _nbytes(*self.h_in)
        self.d2h = _nbytes(self.h_out)
        self.set_bytes = per_set

    def step(self, i=0):
        x, z, out = self.sets[i % self.R]
        self.hb.delta_gated_norm(self.shape, x, z, self.weight, out, rows=self.rows, eps=1e-6)

    def e2e_step(self, i=0):
        x, z, out = self.sets[0]
        for d, h in zip((x, z), self.h_in):
            d.copy_(h, non_blocking=True)
        self.step(0)
        self.h_out.copy_(out, non_blocking=True)



SNAP_LAYERS, SNAP_EVERY, SNAP_POS = 32, 4, 32768  # every 4th layer full attention
SNAP_VOCAB = 248_320


class SnapshotWorkload(Workload):
    """One sequence's state at SNAP_POS positions: the KV of the full-attention
    layers (Hkv 4, d 256, reserve SNAP_POS), the DeltaNet conv and recurrent
    states of the others, the logits; a step is one hb_snapshot_take into a
    pinned host image in the reference's format.  The host link's rate is
    measured in the same run by one contiguous pinned copy of the same size."""
    graphable = False  # the take writes the image's header on the host
    launches_per_step = 0  # copies only: 2 per attention layer (K, V) + 3 (states, logits)

    def __init__(self, device, seed=0x5EED0009):
        import numpy as np
        import torch
        import herbert_b200 as hb
        self.hb = hb
        gen = torch.Generator(device=device).manual_seed(seed)
        hds = [HD if l % SNAP_EVERY == SNAP_EVERY - 1 else 0 for l in range(SNAP_LAYERS)]
        n_delta = hds.count(0)
        offsets = np.concatenate([[0], np.cumsum([2 * HKV * SNAP_POS * h for h in hds])])
        conv = n_delta * (2 * NK * HKD + NV * HVD) * 4
        rec = n_delta * NV * HKD * HVD
        logits = -(-SNAP_VOCAB // 16) * 16
        self.geo = hb.Geometry(offsets, HKV, SNAP_POS, conv, rec, logits)
        self.kv = torch.randint(-32768, 32767, (int(offsets[-1]),), dtype=torch.int16,
                                device=device, generator=gen)
        self.conv = torch.randn(conv, generator=gen, device=device)
        self.rec = torch.randn(rec, generator=gen, device=device)
        self.logits = torch.randint(-32768, 32767, (logits,), dtype=torch.int16, device=device,
                                    generator=gen)
        self.nbytes = hb.snapshot_bytes(self.geo, SNAP_POS)
        self.image = torch.empty(self.nbytes, dtype=torch.uint8).pin_memory()
        self.flat = torch.empty(int(offsets[-1]) * 2 + conv * 4 + rec * 4 + logits * 2,
                                dtype=torch.uint8, device=device)
        self.work = self.nbytes
        self.units = "GB/s"
        self.R = 1
        self.set_bytes = self.nbytes
        self.h2d = self.nbytes
        self.d2h = self.nbytes

    def step(self, i=0):
        self.hb.snapshot_take(self.geo, self.kv, self.conv, self.rec, self.logits, self.image,
                              pos=SNAP_POS, max_positions=SNAP_POS)

    def e2e_step(self, i=0):
        self.step(i)
        self.hb.snapshot_restore(self.geo, self.kv, self.conv, self.rec, self.logits, self.image,
                                 p=SNAP_POS)

    def kernel_probe(self, reps=3):
        """(bytes, seconds) of one take, and the rate of a contiguous pinned
        device-to-host copy of the same bytes (the host link's ceiling)."""
        import torch
        st = torch.cuda.current_stream()

        def timed(fn):
            fn()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            a.record(st)
            for _ in range(reps):
                fn()
            b.record(st)
            torch.cuda.synchronize()
            return a.elapsed_time(b) / 1e3 / reps

        t_take = timed(self.step)
        t_flat = timed(lambda: self.image[:self.flat.numel()].copy_(self.flat, non_blocking=True))
        self.link_gbs = self.flat.numel() / t_flat / 1e9
        return self.nbytes, t_take



def mixer_step_bytes(pos=SNAP_POS):
    """Algorithmic bytes of one decode token through the hybrid model's mixers:
    per attention layer the K and V read (pos + 1 positions), the new k and v
    written, q and gate read and q written back, the output written; per
    DeltaNet layer the recurrent state read and written, the conv state read
    and written with its weights, the qkv row read and written, ab, z read,
    the bf16 output written."""
    n_attn = SNAP_LAYERS // SNAP_EVERY
    n_delta = SNAP_LAYERS - n_attn
    n = pos + 1
    attn = 2 * HKV * n * HD * 2 + 2 * HKV * HD * 2 * 2 + 2 * HQ * HD * 2 + HQ * HD * 2 * 2
    conv = 2 * NK * HKD + NV * HVD
    delta = (2 * NV * HKD * HVD * 4 + conv * 4 * (4 * 2 + 2) + conv * 4 * 2 + 2 * NV * 4
             + NV * HVD * 4 + NV * HVD * 2)
    return n_attn * attn + n_delta * delta


class MixersWorkload(Workload):
    """One decode token through every layer's mixer of a 32-layer hybrid
    (every 4th layer full attention over SNAP_POS cached positions, the others
    DeltaNet), routed by an hb_mount; one CUDA graph holds the 32 mixer calls."""

    def __init__(self, device, seed=0x5EED000A):
        import numpy as np
        import torch
        import herbert_b200 as hb
        self.hb = hb
        gen = torch.Generator(device=device).manual_seed(seed)
        kinds = [hb.HB_LAYER_ATTENTION if l % SNAP_EVERY == SNAP_EVERY - 1 else hb.HB_LAYER_DELTA
                 for l in range(SNAP_LAYERS)]
        self.kinds = kinds
        n_delta = kinds.count(hb.HB_LAYER_DELTA)
        res = SNAP_POS
        offsets = np.concatenate([[0], np.cumsum([2 * HKV * res * HD if k == hb.HB_LAYER_ATTENTION
                                                  else 0 for k in kinds])])
        conv = 2 * NK * HKD + NV * HVD
        self.geo = hb.Geometry(offsets, HKV, res, n_delta * conv * 4, n_delta * NV * HKD * HVD, 16)
        self.kv = _randn_bf16((int(offsets[-1]),), gen, device)
        self.dn_conv = torch.randn(n_delta * conv * 4, generator=gen, device=device)
        self.dn_rec = 0.05 * torch.randn(n_delta * NV * HKD * HVD, generator=gen, device=device)
        self.logits = torch.zeros(16, dtype=torch.bfloat16, device=device)
        half = 32
        pos = torch.arange(res, dtype=torch.float64, device=device)[:, None]
        inv = 1e7 ** (-torch.arange(half, dtype=torch.float64, device=device) * 2 / 64)
        self.cos = torch.cos(pos * inv).to(torch.bfloat16)
        self.sin = torch.sin(pos * inv).to(torch.bfloat16)
        desc, keep = hb.mount_desc(
            self.geo, kinds, kv=self.kv, dn_conv=self.dn_conv, dn_recurrent=self.dn_rec,
            logits=self.logits, attn=hb.attention_spec(HQ, HQ // HKV, HD, True),
            attn_scale=1.0 / 16, rotary=64, cos=self.cos, sin=self.sin, norm_eps=1e-6,
            gemma=True, delta=hb.DeltaShape(nk=NK, nv=NV, hkd=HKD, hvd=HVD), conv_kernel=4,
            conv_stride=conv * 4, recurrent_stride=NV * HKD * HVD, max_rows=1)
        self.mount = hb.Mount(desc, keep)
        qd = HQ * HD
        self.q = _randn_bf16((1, 2 * qd), gen, device)
        self.k = _randn_bf16((1, HKV * HD), gen, device)
        self.v = _randn_bf16((1, HKV * HD), gen, device)
        self.q_norm = (0.1 * torch.randn(HD, generator=gen, device=device)).to(torch.bfloat16)
        self.k_norm = (0.1 * torch.randn(HD, generator=gen, device=device)).to(torch.bfloat16)
        self.attn_out = torch.empty((1, qd), dtype=torch.bfloat16, device=device)
        self.qkv = torch.randn((1, conv), generator=gen, device=device)
        self.ab = 2.0 * torch.randn((1, 2 * NV), generator=gen, device=device)
        self.z = torch.randn((1, NV * HVD), generator=gen, device=device)
        self.conv_w = (0.25 * torch.randn((conv, 4), generator=gen, device=device)).to(
            torch.bfloat16)
        dt = torch.exp(torch.empty(NV, device=device).uniform_(-6.9, -2.3, generator=gen))
        self.dt_bias = (dt + torch.log(-torch.expm1(-dt))).to(torch.bfloat16)
        self.a_log = torch.log(torch.empty(NV, device=device).uniform_(1.0, 16.0, generator=gen))
        self.norm_w = (1.0 + 0.1 * torch.randn(HVD, generator=gen, device=device)).to(
            torch.bfloat16)
        self.delta_out = torch.empty((1, NV * HVD), dtype=torch.bfloat16, device=device)
        self.work = 1  # tokens
        self.units = "tok/s"
        self.bytes_per_step = mixer_step_bytes()
        self.R = 1
        self.set_bytes = self.bytes_per_step
        # one launch per layer: the one-row attention layer over SNAP_POS
        # positions runs its front end inside the decode launch, the one-row
        # DeltaNet layer is one fused launch
        self.launches_per_step = SNAP_LAYERS
        self.h_in = [self.q.cpu().pin_memory(), self.qkv.cpu().pin_memory()]
        self.h_out = [torch.empty(t.shape, dtype=t.dtype).pin_memory()
                      for t in (self.attn_out, self.delta_out)]
        self.h2d = _nbytes(*self.h_in)
        self.d2h = _nbytes(*self.h_out)

    def step(self, i=0):
        pos = SNAP_POS - 1
        for layer, kind in enumerate(self.kinds):
            if kind == self.hb.HB_LAYER_ATTENTION:
                self.mount.attention(layer, self.q, self.k, self.v, self.q_norm, self.k_norm,
                                     self.attn_out, rows=1, pos=pos)
            else:
                self.mount.delta(layer, self.qkv, self.ab, self.z, self.conv_w, self.dt_bias,
                                 self.a_log, self.norm_w, self.delta_out, rows=1)

    def e2e_step(self, i=0):
        for d, h in zip((self.q, self.qkv), self.h_in):
            d.copy_(h, non_blocking=True)
        self.step(i)
        for h, d in zip(self.h_out, (self.attn_out, self.delta_out)):
            h.copy_(d, non_blocking=True)



def config_of(cfg, world):
    """The `config` object of the JSON line; both arms print the same one."""
    attn = {"q_heads": HQ, "kv_heads": HKV, "head_dim": HD, "gate": "sigmoid"}
    delta = {"key_heads": NK, "value_heads": NV, "head_k_dim": HKD, "head_v_dim": HVD}
    rotated = ("inputs rotate over copies totalling more than twice the 126 MB L2, so every "
               "step reads cold inputs")
    if cfg == "prefill":
        d = dict(workload="causal prefill SDPA (BASELINE configs[1])", seq_len=PREFILL_S,
                 past=0, **attn, l2=rotated)
    elif cfg == "decode":
        d = dict(workload="single decode step gated SDPA" + (" (BASELINE configs[0])" if DECODE_N == 2048 else f" over {DECODE_N} cached positions"),
                 kv_len=DECODE_N, **attn, l2=rotated)
    elif cfg == "gdn":
        d = dict(workload="GatedDeltaNet prefill then decode (BASELINE configs[2])",
                 prefill_tokens=GDN_T, decode_steps=GDN_STEPS, **delta, l2=rotated)
    elif cfg == "batch":
        d = dict(workload="batched decode SDPA, sequences sharded by the library's plan "
                 "(BASELINE configs[3])", sequences=64, kv_len="U{1024..32768} seed 0x5EED0004",
                 **attn, l2="inputs larger than L2: every step streams all caches of the GPU "
                 "(4.4 GB in all)")
    elif cfg == "cp":
        d = dict(workload="long-context causal prefill SDPA (BASELINE configs[4])",
                 seq_len=CP_S, **attn, chunk=CP_S // (2 * world),
                 l2="inputs larger than L2: each GPU reads at least 0.3 GB of q, K and V per "
                 "step (2.7 GB on one GPU)")
    elif cfg == "cp_hops":
        d = dict(workload="one rank's hops of an emulated context-parallel ring on one GPU "
                 "(the hop kernel of BASELINE configs[4])", seq_len=CP_S, **attn,
                 ring_ranks=CP_HOPS_RANKS, rank=CP_HOPS_RANK, chunk=cp_hops_chunk(),
                 l2="inputs larger than L2 (q rows 268 MB, 8 shards of 67 MB at chunk 8192)")
    elif cfg == "front":
        d = dict(workload="attention front end: q/k GemmaRMSNorm head norms + partial RoPE "
                 "(64 of 256) + KV append, one 4096-row block", rows=PREFILL_S,
                 q_heads=HQ, kv_heads=HKV, head_dim=HD, rotary=FRONT_ROTARY, l2=rotated)
    elif cfg == "gdn_front":
        d = dict(workload="DeltaNet front end: causal depthwise conv (K 4) + SiLU over the "
                 "qkv projection in place, beta/decay gates; one 4096-row block", rows=GDN_T,
                 **delta, conv_channels=2 * NK * HKD + NV * HVD, l2=rotated)
    elif cfg == "gdn_norm":
        d = dict(workload="DeltaNet gated RMS norm: y = rmsnorm(x) w silu(z) per V head, bf16 "
                 "out; one 4096-row block", rows=GDN_T, value_heads=NV, head_v_dim=HVD,
                 l2=rotated)
    elif cfg == "snapshot":
        d = dict(workload="snapshot of one sequence's state (reference Instantaneous format) "
                 "into a pinned host image", positions=SNAP_POS, layers=SNAP_LAYERS,
                 attention_layers=SNAP_LAYERS // SNAP_EVERY, kv_heads=HKV, head_dim=HD,
                 deltanet_layers=SNAP_LAYERS - SNAP_LAYERS // SNAP_EVERY,
                 l2="the 1.1 GB state is larger than L2")
    elif cfg == "mixers":
        d = dict(workload="one decode token through the mixers of a 32-layer hybrid model "
                 "routed by hb_mount (projections excluded)", positions=SNAP_POS,
                 attention_layers=SNAP_LAYERS // SNAP_EVERY,
                 deltanet_layers=SNAP_LAYERS - SNAP_LAYERS // SNAP_EVERY, **attn,
                 value_heads=NV, head_k_dim=HKD, bytes_per_token=mixer_step_bytes(),
                 l2="8 caches of 134 MB and 24 DeltaNet states per token, larger than L2")
    else:
        raise SystemExit(f"unknown config {cfg}")
    if cfg == "batch":
        par = f"sequences sharded over {world} GPUs, no collective"
    elif cfg == "cp":
        par = (f"context parallel over {world} GPUs: zig-zag shards, K/V ring by NCCL "
               "send/recv, log-sum-exp merge" if world > 1 else "one GPU, whole sequence")
    else:
        par = f"{world} independent replicas"
    d["parallelism"] = par
    return d


METRIC = {"prefill": "prefill SDPA TFLOP/s", "decode": "attn decode HBM GB/s",
          "gdn": "GDN tok/s", "batch": "attn decode HBM GB/s", "cp": "prefill SDPA TFLOP/s",
          "cp_hops": "prefill SDPA TFLOP/s",
          "front": "attn front end HBM GB/s", "gdn_front": "GDN front end HBM GB/s",
          "gdn_norm": "GDN gated norm HBM GB/s", "snapshot": "snapshot take GB/s",
          "mixers": "mixer decode tok/s"}
BOUND = {"prefill": "tensor", "decode": "hbm", "gdn": "tensor", "batch": "hbm", "cp": "tensor",
         "cp_hops": "tensor",
         "front": "hbm", "gdn_front": "hbm", "gdn_norm": "hbm", "snapshot": "host link",
         "mixers": "hbm"}
STRONG = ("batch", "cp")  # total work fixed as the GPUs grow


def make_workload(cfg, device, rank, world):
    if cfg == "prefill":
        return PrefillWorkload(device)
    if cfg == "decode":
        return DecodeWorkload(device)
    if cfg == "gdn":
        return GdnWorkload(device)
    if cfg == "batch":
        return BatchWorkload(device, rank, world)
    if cfg == "cp":
        return CpWorkload(device, rank, world)
    if cfg == "cp_hops":
        return CpHopsWorkload(device)
    if cfg == "front":
        return FrontWorkload(device)
    if cfg == "gdn_front":
        return GdnFrontWorkload(device)
    if cfg == "gdn_norm":
        return GdnNormWorkload(device)
    if cfg == "snapshot":
        return SnapshotWorkload(device)
    if cfg == "mixers":
        return MixersWorkload(device)
    raise SystemExit(f"unknown config {cfg}")


def value_of(work, seconds, units):
    if units == "TFLOP/s":
        return work / seconds / 1e12
    if units == "GB/s":
        return work / seconds / 1e9
    return work / seconds


# ---------------------------------------------------------------- GPU arm

def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600),
                                device_id=device)
    cfg = args.config
    wl = make_workload(cfg, device, rank, world)
    stream = torch.cuda.current_stream()

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for i in range(args.warmup):
        wl.step(i)
        wl.e2e_step(i)
    barrier()

    def capture(fn, steps):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(steps):
                fn(i)
        return g

    def timed(graph):
        graph.replay()  # untimed replay: the graph's first launch uploads it
        torch.cuda.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        graph.replay()
        b.record(stream)
        torch.cuda.synchronize()
        return a.elapsed_time(b) / 1e3  # seconds for all steps

    def timed_eager(fn):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for i in range(args.steps):
            fn(i)
        b.record(stream)
        torch.cuda.synchronize()
        return a.elapsed_time(b) / 1e3

    if wl.graphable:
        g_dev = capture(wl.step, args.steps)
        g_e2e = capture(wl.e2e_step, args.steps)
        run_dev, run_e2e = (lambda: timed(g_dev)), (lambda: timed(g_e2e))
    else:
        run_dev, run_e2e = (lambda: timed_eager(wl.step)), (lambda: timed_eager(wl.e2e_step))
    barrier()
    sampler = ClockSampler(smi_index(local)).start() if rank == 0 else None
    t_dev = run_dev()
    barrier()
    clocks = sampler.stop() if sampler else None
    t_e2e = run_e2e()
    barrier()
    probe = wl.kernel_probe() if hasattr(wl, "kernel_probe") else None
    barrier()
    if wl.graphable:
        del g_dev, g_e2e

    t = torch.tensor([t_dev, t_e2e], dtype=torch.float64, device=device)
    work = torch.tensor([float(wl.work)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(work, op=dist.ReduceOp.SUM)
    t_dev, t_e2e = float(t[0]), float(t[1])
    total_work = float(work[0])

    if rank == 0:
        pk = peaks()
        per_launch = wl.work
        kernel_s = t_dev / args.steps
        # a dense kernel kept busy for half a second or more runs at the power
        # cap: its denominator is the sustained GEMM figure, else the burst one
        sustained = t_dev >= 0.5
        bf16_peak = pk["bf16_sustained"] if sustained else pk["bf16"]
        if probe is not None and cfg == "snapshot":
            achieved = probe[0] / probe[1] / 1e9
            peak, unit = round(wl.link_gbs, 3), "GB/s"
        elif probe is not None:
            achieved = probe[0] / probe[1] / 1e12
            peak, unit = bf16_peak, "TFLOP/s"
        elif BOUND[cfg] == "tensor":
            achieved = per_launch / kernel_s / 1e12
            peak, unit = bf16_peak, "TFLOP/s"
        elif cfg == "mixers":
            achieved = wl.bytes_per_step / kernel_s / 1e9
            peak, unit = pk["hbm"], "GB/s"
        else:
            achieved = per_launch / kernel_s / 1e9
            peak, unit = pk["hbm"], "GB/s"
        line = {
            "metric": METRIC[cfg],
            "value": round(value_of(total_work, t_dev / args.steps, wl.units), 4),
            "unit": wl.units,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(t_dev / args.steps * 1e3, 5),
            "higher_is_better": True,
            "scaling": "strong" if cfg in STRONG else "weak",
            "vs_baseline": None,
            "dtype": ("f32" if cfg in ("gdn", "gdn_front", "gdn_norm") else
                      "bytes" if cfg == "snapshot" else
                      "bf16 attention, f32 DeltaNet" if cfg == "mixers" else "bf16"),
            "data": "synthetic",
            "config": config_of(cfg, world),
            "timing": (f"one CUDA graph of {args.steps} steps between CUDA events"
                       if wl.graphable else
                       f"{args.steps} steps issued eagerly between CUDA events") + (
                           f"; inputs rotate over {wl.R} copies "
                           f"({wl.R * wl.set_bytes / 2**20:.0f} MiB) per GPU" if wl.R > 1 else ""),
            "roofline": {"bound": BOUND[cfg], "achieved": round(achieved, 3), "peak": peak,
                         "unit": unit, "frac": round(achieved / peak, 4),
                         "peak_source": pk["source"] + (
                             ("" if unit != "TFLOP/s" else
                              " sustained (timed region >= 0.5 s)" if sustained else " burst")),
                         "traffic": None if (cfg == "cp" and world > 1) or (cfg == "decode" and DECODE_N != 2048)
                                    else NCU_TRAFFIC.get(cfg)},
            "e2e": {"value": round(value_of(total_work, t_e2e / args.steps, wl.units), 4),
                    "unit": wl.units, "h2d_bytes_per_step": int(wl.h2d),
                    "d2h_bytes_per_step": int(wl.d2h)},
            "gpu_launches": int(wl.launches_per_step * args.steps),
            **({"dma_copies": (2 * (SNAP_LAYERS // SNAP_EVERY) + 3) * args.steps}
               if cfg == "snapshot" else {}),
            "clocks": clocks,
        }
        if probe is not None:
            line["roofline"]["kernel"] = (
                "gdn_prep_kernel + gdn_scan_kernel (one chunked prefill of T tokens)"
                if cfg == "gdn" else
                "hb_snapshot_take: one 2-D copy per (layer, K|V) and one per state"
                if cfg == "snapshot" else
                "attn_prefill_kernel over the whole sequence" if world == 1 else
                "attn_prefill_kernel<CP> hop over the rank's own shard (hop 0)")
            line["roofline"]["launch_ms"] = round(probe[1] * 1e3, 4)
            if cfg == "snapshot":
                line["roofline"]["peak_source"] = ("a contiguous pinned device-to-host copy of "
                                                   "the same bytes, measured in this run")
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(cfg, budget_s=args.cpu_seconds)
        print(json.dumps(line), flush=True)
    if hasattr(wl, "close"):
        wl.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------- CPU arm

def _cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_baseline(cfg, budget_s=10.0, threads=0):
    """Times the oracle (the C restatement of the reference's x86 kernels)
    on this host's cores over a bounded sample of the configuration."""
    sys.path[:0] = [os.path.join(ROOT, "oracle")]
    import numpy as np
    import oracle
    from herbert_b200.inputs import AttentionInputs, DeltaInputs

    oracle.build()
    threads = threads or _cpu_threads()
    impl = 1 if oracle.has_avx512bf16() else 0
    if cfg in ("prefill", "cp", "cp_hops"):
        S = PREFILL_S if cfg == "prefill" else CP_S
        rows = (256 if impl else 32) if cfg == "prefill" else (16 if impl else 2)
        past = S - rows
        inp = AttentionInputs(rows, past)
        work = prefill_flops(rows, past)
        unit, scale = "TFLOP/s", 1e12
        sample = f"last {rows} rows of the S={S} prefill (all 16 heads)"
        fn = lambda: oracle.attention(  # noqa: E731
            inp.q.ravel(), inp.keys.ravel(), inp.values.ravel(), rows=rows, past=past,
            heads=HQ, gqa=HQ // HKV, head_dim=HD, q_row=inp.q_row, q_head=HD,
            out_row=inp.out_row, gate_offset=inp.gate_offset, kv_stride=inp.kv_stride,
            scale=inp.scale, impl=impl, use_block=0 if impl else 1, threads=threads)
    elif cfg in ("decode", "batch"):
        n = DECODE_N if cfg == "decode" else 16896
        inp = AttentionInputs(1, n - 1)
        work = 2 * HKV * n * HD * 2 + 3 * HQ * HD * 2
        unit, scale = "GB/s", 1e9
        sample = f"one decode step at n={n}" + (" (the mean batch length)" if cfg == "batch" else "")
        fn = lambda: oracle.attention(  # noqa: E731
            inp.q.ravel(), inp.keys.ravel(), inp.values.ravel(), rows=1, past=n - 1,
            heads=HQ, gqa=HQ // HKV, head_dim=HD, q_row=inp.q_row, q_head=HD,
            out_row=inp.out_row, gate_offset=inp.gate_offset, kv_stride=inp.kv_stride,
            scale=inp.scale, impl=impl, use_block=0, threads=threads)
    elif cfg == "front":
        from herbert_b200.inputs import FrontInputs
        rows = 256
        f = FrontInputs(rows, 0, capacity=rows)
        work = front_bytes(rows)
        unit, scale = "GB/s", 1e9
        sample = f"{rows} rows of the 4096-row block (one thread)"
        threads = 1
        fn = lambda: oracle.attn_front(  # noqa: E731
            f.q, f.k, f.v, f.q_norm, f.k_norm, f.cos, f.sin, heads=HQ, kv_heads=HKV,
            head_dim=HD, rotary=FRONT_ROTARY, past=0, keys=f.keys, values=f.values, impl=impl)
    elif cfg in ("gdn_front", "gdn_norm"):
        from herbert_b200.inputs import DeltaFrontInputs
        rows = 256
        d = DeltaFrontInputs(rows)
        unit, scale = "GB/s", 1e9
        threads = 1
        sample = f"{rows} rows of the 4096-row block (one thread)"
        if cfg == "gdn_front":
            work = gdn_front_bytes(rows)

            def fn():
                oracle.gdn_conv(d.qkv, d.conv_state, d.conv_weight, impl)
                oracle.gdn_gates(d.ab, d.dt_bias, d.a_log)
        else:
            work = gdn_norm_bytes(rows)
            fn = lambda: oracle.gdn_gated_norm(d.x, d.z, d.norm_weight, 1e-6, impl)  # noqa: E731
    elif cfg == "mixers":
        from herbert_b200.inputs import DeltaFrontInputs, FrontInputs
        pos = SNAP_POS - 1
        inp = AttentionInputs(1, pos)
        f = FrontInputs(1, pos, capacity=pos + 1)
        d = DeltaFrontInputs(1)
        state = np.zeros((NV, HKD, HVD), np.float32)
        n_attn = SNAP_LAYERS // SNAP_EVERY
        work = 1
        unit, scale = "tok/s", 1.0
        sample = (f"one token through {n_attn} attention mixers at {SNAP_POS} positions and "
                  f"{SNAP_LAYERS - n_attn} DeltaNet mixers, all host threads")

        def fn():
            for _ in range(n_attn):
                oracle.attn_front(f.q, f.k, f.v, f.q_norm, f.k_norm, f.cos, f.sin, heads=HQ,
                                  kv_heads=HKV, head_dim=HD, rotary=FRONT_ROTARY, past=pos,
                                  impl=impl)
                oracle.attention(inp.q.ravel(), inp.keys.ravel(), inp.values.ravel(), rows=1,
                                 past=pos, heads=HQ, gqa=HQ // HKV, head_dim=HD, q_row=inp.q_row,
                                 q_head=HD, out_row=inp.out_row, gate_offset=inp.gate_offset,
                                 kv_stride=inp.kv_stride, scale=inp.scale, impl=impl,
                                 use_block=0, threads=threads)
            for _ in range(SNAP_LAYERS - n_attn):
                y, _ = oracle.gdn_conv(d.qkv, d.conv_state, d.conv_weight, impl)
                b, dc = oracle.gdn_gates(d.ab, d.dt_bias, d.a_log)
                out, _, _ = oracle.gdn_layer(y, state, b, dc, nk=NK, nv=NV, hkd=HKD, hvd=HVD,
                                             threads=threads)
                oracle.gdn_gated_norm(out, d.z, d.norm_weight, 1e-6, impl)
    elif cfg == "snapshot":
        sys.path[:0] = [os.path.join(ROOT, "oracle")]
        import snapshot as S
        hds = [HD if l % SNAP_EVERY == SNAP_EVERY - 1 else 0 for l in range(SNAP_LAYERS)]
        n_delta = hds.count(0)
        r = S.Runner(HKV, SNAP_POS, hds, n_delta * (2 * NK * HKD + NV * HVD) * 4,
                     n_delta * NV * HKD * HVD, -(-SNAP_VOCAB // 16) * 16)
        r.kv[:] = np.arange(r.kv.size, dtype=np.uint64).astype(np.uint16)  # any bits
        r.pos = SNAP_POS
        slot = np.zeros(len(S.image_c(r, SNAP_POS)), np.uint8)  # reserved once
        work = slot.size
        unit, scale = "GB/s", 1e9
        threads = 1
        sample = (f"the same state at {SNAP_POS} positions: the C restatement of take + "
                  "write_to into a slot reserved once (memcpy per head, one thread, as the "
                  "reference copies)")

        def fn():
            S.image_c(r, SNAP_POS, out=slot)
    else:  # gdn
        T = 64
        d = DeltaInputs(T)
        work = T
        unit, scale = "tok/s", 1.0
        sample = f"{T} positions of the recurrence at Qwen3.5 geometry (32 value heads)"
        fn = lambda: oracle.gdn_layer(d.qkv, d.state, d.beta, d.decay, nk=NK, nv=NV,  # noqa
                                      hkd=HKD, hvd=HVD, threads=threads)
    fn()  # warm
    reps, t0 = 0, time.perf_counter()
    while True:
        fn()
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or reps >= 100000:
            break
    val = work * reps / el / scale
    return {"value": round(val, 6), "unit": unit, "cores": threads,
            "kind": "port",
            "sample": sample + f", repeated {reps}x in {el:.1f} s" + (
                "" if cfg in ("snapshot",) else
                f"; {'AVX512-BF16 transcription' if impl else 'portable emulation'}")}


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg = args.config
    budget = max(1.0, min(20.0, 60.0 / max(1, args.steps + args.warmup)))
    for _ in range(args.warmup):
        cpu_baseline(cfg, budget_s=0.2)
    vals = [cpu_baseline(cfg, budget_s=budget) for _ in range(args.steps)]
    v = statistics.median(x["value"] for x in vals)
    base = vals[0]
    line = {
        "impl": "reference",
        "metric": METRIC[cfg], "value": v, "unit": base["unit"], "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "scaling": "strong" if cfg in STRONG else "weak", "vs_baseline": None,
        "dtype": ("f32" if cfg in ("gdn", "gdn_front", "gdn_norm") else
                  "bytes" if cfg == "snapshot" else
                  "bf16 attention, f32 DeltaNet" if cfg == "mixers" else "bf16"),
        "data": "synthetic",
        "config": config_of(cfg, world),
        "note": ("CPU restatement of the reference's x86 AVX-512 BF16 kernels (the Rust "
                 "reference cannot be built here); rank 0 alone runs it"),
        "cpu_baseline": dict(base, value=v),
        "e2e": {"value": v, "unit": base["unit"], "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _free_port():
    import socket
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="cp", choices=sorted(METRIC))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.gpus < 1:
        raise SystemExit("--gpus must be at least 1")
    if "WORLD_SIZE" not in os.environ and args.gpus > 1:
        # not under torchrun: start one rank per GPU on this node
        cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
               f"--nproc-per-node={args.gpus}", "--master-addr", "127.0.0.1",
               "--master-port", str(_free_port()), os.path.abspath(__file__)] + sys.argv[1:]
        raise SystemExit(subprocess.call(cmd))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but {world} ranks were started")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
