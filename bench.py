"""Benchmark of DPUF's per-token LM loop on B200: Qwen3-8B-shaped random-init mode-12 model,
prompt of 32 ids (pp32) then batch-1 greedy decode (tg).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl dpuf|reference]

A step is one greedy decode token at batch 1 (the reference CLI's decode loop, dpuf-cli.c:2398-2420).
  value   decode tok/s, device time (CUDA events on the engine stream) of K back-to-back steps
          with the token fed back on the device; weights (4.26 GB) exceed L2, so every step
          streams them from HBM
  e2e     the same steps through the reference's C ABI (dpuf_engine_forward_token): token id
          host->device, logits[vocab] device->host, greedy argmax on the host
  roofline  the dominant kernel (the mode-12 decode GEMV, gate/up shape 2x12288x4096) timed alone
          with CUDA events over 8 weight copies (> L2), bytes = tile bytes per launch
  cpu_baseline  the reference's own AVX2/OpenMP engine (built from its sources) on this host's
          cores, same model and prompt, a bounded number of decode steps
Model: the random-init model is written once as a DPUF0001 container by a separate process
(`python -m dpuf_b200.container write`) and both arms map that same file.
Multi-GPU (torchrun, --gpus N): the N ranks decode ONE sequence with tensor parallelism (every
projection and the LM head split over all GPUs' CTAs, outputs exchanged through peer memory
inside the persistent kernel; strong scaling); every rank first records the same sequence on its
GPU alone and the line's tp_parity says whether ids and logits were bit-identical (rank 0 exits
non-zero if not).  With --dp each GPU decodes its own sequence instead (weak scaling).  Times
are the max over ranks.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import pathlib
import statistics
import subprocess
import sys
import threading
import time

REPO = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

import numpy as np  # noqa: E402

PEAKS_FILE = REPO / "MEASURED_PEAKS.json"
FALLBACK_HBM_GBS = 6650.0


def peaks():
    try:
        p = json.loads(PEAKS_FILE.read_text())
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons of one GPU, sampled through NVML every 5 ms
    from a background thread while the timed region runs (plus one sample at its start).  The
    GPU is found by the PCI bus id of the CUDA device, so the sampler follows torchrun's and
    CUDA_VISIBLE_DEVICES' device numbering."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, cuda_index: int):
        self.cuda_index = cuda_index
        self.samples = []  # (sm MHz, reasons bitmask)
        self.max_mhz = None
        self.error = None
        self._stop = threading.Event()
        self._thread = None
        self._nvml = None
        self._h = None

    def _handle(self):
        import pynvml
        import torch

        pynvml.nvmlInit()
        self._nvml = pynvml
        p = torch.cuda.get_device_properties(self.cuda_index)
        bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        try:
            return pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
        except pynvml.NVMLError:
            return pynvml.nvmlDeviceGetHandleByPciBusId(bus)

    def _sample(self):
        nv = self._nvml
        self.samples.append((float(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)),
                             int(nv.nvmlDeviceGetCurrentClocksEventReasons(self._h))))

    def _run(self):
        while not self._stop.wait(0.005):
            try:
                self._sample()
            except Exception as e:  # noqa: BLE001 - a sampling failure must not end the run
                self.error = str(e)
                return

    def __enter__(self):
        try:
            self._h = self._handle()
            self.max_mhz = float(self._nvml.nvmlDeviceGetMaxClockInfo(self._h, self._nvml.NVML_CLOCK_SM))
            self._sample()
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        except Exception as e:  # noqa: BLE001
            self.error = str(e)
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread:
            self._thread.join(timeout=2)
        try:
            if self._h is not None:
                self._sample()
        except Exception:  # noqa: BLE001
            pass

    def summary(self):
        sm = [c for c, _ in self.samples]
        reasons = sorted(n for n, bit in self.REASONS.items() if any(r & bit for _, r in self.samples))
        out = {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz, "reasons": reasons,
               "samples": len(sm), "source": "NVML, 5 ms"}
        if self.error:
            out["error"] = self.error
        return out


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def allreduce_max(x: float, world: int, device: str = "cuda") -> float:
    """Max of x over the ranks of the default process group (device "cpu" for gloo)."""
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def dp_value(local_ms: float, steps: int, world: int, device: str = "cuda"):
    """Data-parallel decode throughput: every rank decodes its own sequence for `steps` steps;
    the job's time is the slowest rank's, the job's tokens are world * steps.  Returns
    (tok/s of the whole job, the max time in ms)."""
    dev_ms = allreduce_max(float(local_ms), world, device)
    return world * steps / (dev_ms * 1e-3), dev_ms


def tp_value(local_ms: float, steps: int, world: int, device: str = "cuda"):
    """Tensor-parallel decode throughput: all ranks decode ONE sequence, so the job's tokens are
    the steps and its time is the slowest rank's.  Returns (tok/s, the max time in ms)."""
    dev_ms = allreduce_max(float(local_ms), world, device)
    return steps / (dev_ms * 1e-3), dev_ms


def parity_agreed(local_ok: bool, world: int, device: str = "cuda") -> bool:
    """True only if every rank's own parity check passed (one failing rank fails them all)."""
    return allreduce_max(0.0 if local_ok else 1.0, world, device) == 0.0


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def gemv_roofline(hbm_peak: float, peak_kind: str):
    """Kernel-only timing of the mode-12 decode GEMV on the gate/up shape."""
    import torch

    from dpuf_b200 import engine, model as mdl, packer

    lib = engine.cuda_lib()
    w = packer.gen_normal_bf16(11, 22, (24576, 4096), 0.02)
    bv = packer.BlobView(packer.encode_mode12(w, "blk.0.mlp_in"))
    d = mdl.DpufWeightDesc(12, bv.rows, bv.cols, bv.n_tiles, bv.tiles.ctypes.data, bv.tile_offsets.ctypes.data, None,
                           bv.sign_bits.ctypes.data)
    n_copies = 6  # 6 x 56.7 MB > 126 MB L2
    hs = [lib.dpuf_cuda_w12_upload(ctypes.byref(d)) for _ in range(n_copies)]
    if not all(hs):
        raise RuntimeError(engine.last_error())
    x = torch.randn(1, 4096, device="cuda")
    y = torch.empty(1, 24576, device="cuda")
    arr = (ctypes.c_void_p * n_copies)(*hs)
    ms = ctypes.c_float()
    st = torch.cuda.current_stream().cuda_stream
    rc = lib.dpuf_cuda_matmul_dev_timed(arr, n_copies, 1, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()),
                                        60, ctypes.c_void_p(st), ctypes.byref(ms))
    for h in hs:
        lib.dpuf_cuda_w12_free(h)
    if rc != 0:
        raise RuntimeError(engine.last_error())
    bytes_per_launch = int(bv.tiles.nbytes)
    achieved = bytes_per_launch / (ms.value * 1e-3) / 1e9
    traffic = None
    prof = REPO / "profiles" / "gemv_m1_gate_up_24576x4096.md"
    if prof.exists():
        for line in prof.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                try:
                    traffic = int(line.split(":", 1)[1].strip())
                except ValueError:
                    pass
    return {"kernel": "gemv_kernel (mode-12 M=1, 24576x4096)", "bound": "hbm", "achieved": round(achieved, 1),
            "peak": hbm_peak, "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
            "traffic": traffic, "bytes_per_launch": bytes_per_launch, "us_per_launch": round(ms.value * 1e3, 2)}


def run_op_configs(hbm_peak: float, peak_kind: str):
    """Config 2 (isolated op): gate-shaped 12288x4096 and down-shaped 4096x12288 mode-12
    matrices at M = 1 (GB/s of tile bytes) and M = 8 / 32 / 64 / 256 (dense-4-bit-equivalent TOP/s,
    2*M*N*K, and the GB/s of the expanded copy the tensor-core GEMM streams), kernel-only timing
    over copies that together exceed L2."""
    import torch

    from dpuf_b200 import engine, packer

    lib = engine.cuda_lib()
    for rows, cols, name in ((12288, 4096, "blk.0.mlp_in"), (4096, 12288, "blk.0.ffn_down.weight")):
        w = packer.gen_normal_bf16(31, rows, (rows, cols), 0.02)
        bv = packer.BlobView(packer.encode_mode12(w, name))
        n_copies = 8  # 8 x 28.4 MB > 126 MB L2
        hs = [engine.upload(bv) for _ in range(n_copies)]
        arr = (ctypes.c_void_p * n_copies)(*hs)
        x = torch.randn(256, cols, device="cuda")
        if "down" in name:
            x[x.abs() < 0.3] = 0.0
        y = torch.empty(256, rows, device="cuda")
        for M in (1, 8, 32, 64, 256):
            ms = ctypes.c_float()
            rc = lib.dpuf_cuda_matmul_dev_timed(arr, n_copies, M, ctypes.c_void_p(x.data_ptr()),
                                                ctypes.c_void_p(y.data_ptr()), 40,
                                                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
                                                ctypes.byref(ms))
            if rc != 0:
                raise RuntimeError(engine.last_error())
            s = ms.value * 1e-3
            line = {"config": "op", "shape": f"{rows}x{cols}", "seed_name": name, "M": M,
                    "us_per_call": round(s * 1e6, 2), "tile_bytes": int(bv.tiles.nbytes)}
            if M == 1:
                gbs = bv.tiles.nbytes / s / 1e9
                line.update({"GB/s": round(gbs, 1), "frac_hbm": round(gbs / hbm_peak, 4), "peak_kind": peak_kind})
            else:
                tc = os.environ.get("DPUF_CUDA_TC_GEMM", "1") != "0"
                x8 = tc and os.environ.get("DPUF_CUDA_TC_EXPAND", "1") != "0"
                # the expanded copy: per 128-row group and 32-column block, 4096 B of s8 weights
                # and 256 B of row scales
                x8_bytes = (bv.n_tiles + 7) // 8 * (cols // 32) * 4352
                line.update({"TOP/s_4bit_equiv": round(2 * M * rows * cols / s / 1e12, 2),
                             "GB/s": round(bv.tiles.nbytes / s / 1e9, 1),
                             "kernel": ("gemm_x8_kernel (tcgen05 kind::i8 over the expanded s8 copy, TMEM)" if x8
                                        else "gemm_tc_kernel (tcgen05 kind::i8, in-kernel unpack, TMEM)" if tc
                                        else "gemm_exact_kernel (dp4a)")})
                if x8:
                    line.update({"expanded_bytes": x8_bytes, "GB/s_expanded": round(x8_bytes / s / 1e9, 1),
                                 "frac_hbm_expanded": round(x8_bytes / s / 1e9 / hbm_peak, 4)})
            print(json.dumps(line), flush=True)
        for h in hs:
            engine.w12_free(h)


def run_had_op_configs(hbm_peak: float, peak_kind: str):
    """Modes 13 / 14 (standalone matmul, dpuf_cuda_had_asym_timed): the gate-shaped 12288x4096
    matrix at M = 1 (GB/s of tile bytes against the copy bandwidth) and M = 32, kernel-only
    timing over copies that together exceed L2."""
    from dpuf_b200 import engine, packer

    lib = engine.cuda_lib()
    lib.dpuf_cuda_had_asym_timed.argtypes = [ctypes.c_int32] * 5 + [ctypes.c_void_p] * 4 + [ctypes.c_int32] * 2 + \
        [ctypes.c_void_p]
    rows, cols = 12288, 4096
    for mode in (13, 14):
        tiles, offs, signs = packer.synth_had_tiles(rows, cols, mode, 7 + mode)
        n_copies = 6  # 6 x 28.3 MB (mode 13) or 6 x 40.9 MB (mode 14) > 126 MB L2
        x = np.random.default_rng(mode).standard_normal((32, cols)).astype(np.float32)
        for M in (1, 32):
            ms = ctypes.c_float()
            rc = lib.dpuf_cuda_had_asym_timed(mode, M, rows, cols, offs.size, x.ctypes.data, tiles.ctypes.data,
                                              offs.ctypes.data, signs.ctypes.data, n_copies, 40, ctypes.byref(ms))
            if rc != 0:
                raise RuntimeError(engine.last_error())
            sec = ms.value * 1e-3
            gbs = tiles.nbytes / sec / 1e9
            line = {"config": "op", "mode": mode, "shape": f"{rows}x{cols}", "M": M,
                    "us_per_call": round(sec * 1e6, 2), "tile_bytes": int(tiles.nbytes), "GB/s": round(gbs, 1),
                    "kernel": "had_gemv_stream_kernel (dp4a, a warp per 8-row group, bulk-copy ring)" if M == 1
                    else "had_asym_kernel (dp4a)", "data": "synthetic codes and scales in the reference layout"}
            if M == 1:
                line.update({"frac_hbm": round(gbs / hbm_peak, 4), "peak_kind": peak_kind})
            else:
                line["TOP/s_equiv"] = round(2 * M * rows * cols / sec / 1e12, 2)
            print(json.dumps(line), flush=True)


def run_zone_config(hbm_peak: float, peak_kind: str, n_vec: int = 4096, za: int = 1000, margin: float = 0.8):
    """Config 4 (Zone-A stress): the 151936x4096 head packed as output.weight, n_vec hidden
    vectors N(0,1), half of them planted with beta * (dequantised head row i), i < 16Z."""
    from dpuf_b200 import engine, packer

    rows, cols = 151936, 4096
    w = packer.gen_normal_bf16(41, 9, (rows, cols), 0.02)
    bv = packer.BlobView(packer.encode_mode12(w, "output.weight"))
    rng = np.random.default_rng(0)
    planted = rng.integers(0, 16 * za, size=n_vec // 2).astype(np.int32)
    x = rng.standard_normal((n_vec, cols)).astype(np.float32)
    x[: n_vec // 2] += np.float32(5.0) * engine.embed(bv, planted)
    engine.zone_head(bv, x[:64], za, margin)  # warm-up
    ids, exits, ms = engine.zone_head(bv, x, za, margin)
    s = ms * 1e-3
    n_exit = int(exits.sum())
    zone_bytes = bv.tiles.nbytes * min(16 * za, rows) / rows
    bytes_total = n_exit * zone_bytes + (n_vec - n_exit) * bv.tiles.nbytes
    print(json.dumps({"config": "zone_a", "head": f"{rows}x{cols}", "zone_tiles": za, "margin": margin,
                      "vectors": n_vec, "vectors_per_s": round(n_vec / s, 1), "exit_fraction": round(n_exit / n_vec, 4),
                      "planted_exit_fraction": round(float(exits[: n_vec // 2].mean()), 4),
                      "planted_id_hits": round(float((ids[: n_vec // 2] == planted).mean()), 4),
                      "GB/s": round(bytes_total / s / 1e9, 1), "frac_hbm": round(bytes_total / s / 1e9 / hbm_peak, 4),
                      "peak_kind": peak_kind, "us_per_vector": round(s / n_vec * 1e6, 2)}), flush=True)


def run_serve_config(args, hbm_peak: float, peak_kind: str, world: int = 1, rank: int = 0, local: int = 0):
    """Config 5 (batched serving): the 8B-shaped model, n_seq independent sequences with
    random prompt_len-token prompts (seed 1000 + i), each prefilled into its own slot in
    256-token forward_batch calls, then `steps` greedy decode steps of all sequences at once
    (the first `warmup` of them untimed)
    through dpuf_cuda_decode_batch (one CUDA-graph launch per step, ids in, ids out).  The
    timed region is the decode steps only; each call is synchronous, so the time is wall clock
    around them (which is also the end-to-end time: it includes the per-step id copies).  Under
    torchrun every rank serves its own n_seq sequences (prompt seeds 1000 + rank * n_seq + i) on
    its GPU, data parallel: the job's tokens are world * n_seq * steps and its time the slowest
    rank's (`scaling` "weak")."""
    from dpuf_b200 import engine, model as mdl

    n_seq, plen, steps, warm = args.serve_seqs, args.serve_prompt, args.serve_steps, args.warmup
    shape = mdl.QWEN3_8B
    if plen + steps > shape.max_seq:
        raise SystemExit("prompt + steps exceed the 2304-position context")
    steps -= warm  # the first `warm` of the decode steps are untimed
    os.environ["DPUF_CUDA_SLOTS"] = str(max(8, n_seq))
    kv = args.serve_kv
    os.environ["DPUF_CUDA_KV_F16"] = "1" if kv == "f16" else "0"
    m = mdl.SyntheticModel(shape, seed=0)
    m.cfg.kv_type = 1 if kv == "q8" else 0  # the reference's Q8 cache (kv_type 1)
    eng = engine.CudaTransformerEngine(m)
    toks, pos = [], []
    t0 = time.perf_counter()
    for i in range(n_seq):
        pr = mdl.prompt_ids(plen, shape.vocab, 1000 + rank * n_seq + i)
        if eng.set_slot(i) != 0:
            raise RuntimeError(engine.last_error())
        eng.reset_slot(i)
        lg = None
        for c0 in range(0, plen, 256):
            lg = eng.forward_batch(pr[c0:c0 + 256], c0)
        toks.append(int(np.argmax(lg[0])))
        pos.append(plen)
    prefill_s = time.perf_counter() - t0
    slots = list(range(n_seq))
    for _ in range(warm):
        toks = [int(t) for t in eng.decode_batch(slots, toks, pos)]
        pos = [p + 1 for p in pos]
    ctx0 = pos[0]
    barrier(world)
    with ClockSampler(local) as clk:
        t0 = time.perf_counter()
        for _ in range(steps):
            toks = [int(t) for t in eng.decode_batch(slots, toks, pos)]
            pos = [p + 1 for p in pos]
        dt = time.perf_counter() - t0
    eng.close()
    if world > 1:  # the slowest rank's time for every rank's tokens
        value, max_ms = dp_value(dt * 1e3, n_seq * steps, world)
        dt = max_ms * 1e-3
    else:
        value = n_seq * steps / dt
    if rank != 0:
        return
    if args.no_extras:
        cpu = None
    else:
        from oracle import oracle as orc

        cpu = serve_cpu_baseline(m, plen, n_seq, 4, min(32, orc.host_threads()))
    # algorithmic bytes per step: the weights once, plus every sequence's K and V rows
    wbytes = shape.weight_bytes_per_token()
    kvd = shape.kv_dim
    ctx_mean = ctx0 + (steps + 1) / 2.0
    kv_bytes = n_seq * shape.layers * 2 * ctx_mean * kvd * {"f16": 2, "f32": 4, "q8": 1.125}[kv]
    step_s = dt / steps
    print(json.dumps({
        "metric": "batched_decode_tok_per_s", "value": round(value, 1), "unit": "tok/s", "n_gpus": world,
        "steps": steps, "warmup": warm, "ms_per_step": round(step_s * 1e3, 3), "higher_is_better": True,
        "scaling": "weak",
        "config": {"workload": f"{shape.name}-shape batched serving: {n_seq} sequences x {plen}-token prompts, "
                               f"{steps} greedy steps at batch {n_seq}" + (" per GPU" if world > 1 else ""),
                   "parallelism": f"dp{world}" if world > 1 else "single",
                   "kv": {"f16": "fp16", "f32": "fp32", "q8": "q8 (kv_type 1)"}[kv],
                   "context": [ctx0, ctx0 + steps]},
        "step_roofline": {"bytes_per_step": int(wbytes + kv_bytes), "weights": wbytes, "kv": int(kv_bytes),
                          "achieved_gbs": round((wbytes + kv_bytes) / step_s / 1e9, 1),
                          "frac": round((wbytes + kv_bytes) / step_s / 1e9 / hbm_peak, 4), "peak": hbm_peak,
                          "peak_kind": peak_kind},
        "e2e": {"value": round(value, 1), "unit": "tok/s", "h2d_bytes_per_step": n_seq * 20,
                "d2h_bytes_per_step": n_seq * 4, "what": "dpuf_cuda_decode_batch per step, synchronous"},
        "prefill": {"tokens": n_seq * plen, "seconds": round(prefill_s, 1),
                    "tok_per_s": round(n_seq * plen / prefill_s, 1)},
        "cpu_baseline": cpu,
        "clocks": clk.summary(),
    }), flush=True)


def serve_cpu_baseline(m, plen: int, n_seq: int, n_steps: int, threads: int):
    """The reference engine serves sequences one at a time, so its throughput at any batch is its
    batch-1 rate at that context: 2 sequences, each prefilled with a plen-token prompt (untimed)
    and then n_steps greedy steps (timed), extrapolated linearly to the batch."""
    from oracle import oracle as orc

    if not orc.RefEngine.available():
        return None
    ref = orc.RefEngine(m, n_threads=threads)
    steps_done, dt = 0, 0.0
    for i in range(2):
        pr = mdl_prompt(plen, m.shape.vocab, 1000 + i)
        ref.reset()
        lg = None
        for c0 in range(0, plen, 256):
            lg = ref.forward(pr[c0:c0 + 256], c0, 1)
        nxt, pos = int(np.argmax(lg[0])), plen
        t0 = time.perf_counter()
        for _ in range(n_steps):
            nxt = int(np.argmax(ref.forward(np.array([nxt], np.int32), pos, 1)[0]))
            pos += 1
        dt += time.perf_counter() - t0
        steps_done += n_steps
    ref.close()
    kv = "q8 (kv_type 1)" if m.cfg.kv_type == 1 else "fp32 (kv_type 0)"
    return {"value": round(steps_done / dt, 3), "unit": "tok/s", "cores": threads, "kind": "reference",
            "sample": f"2 sequences x ({plen}-token prompt untimed + {n_steps} timed greedy steps), one at a time "
                      f"as the reference serves them, {kv} KV; extrapolated linearly to {n_seq} sequences "
                      f"(same tok/s); reference AVX2/OpenMP engine, {orc.cpu_model_string()}"}


def mdl_prompt(n: int, vocab: int, seed: int):
    from dpuf_b200 import model as mdl

    return mdl.prompt_ids(n, vocab, seed)


TRACE_EVENTS = ["norm1_res", "norm1_chain", "norm1", "qkv", "attn_in", "attn_wait", "attn_rope", "attn_scores",
                "attn_softmax", "attn_pv", "attn", "load_o", "o", "norm2_res", "norm2_chain", "norm2", "gate_up_stages",
                "gate_up", "load_down", "down"]


def run_trace(args):
    """Phase trace of the persistent decode kernel (env DPUF_CUDA_TRACE_DECODE=1): per layer, the
    critical-path time of each consumer phase - the increase of the latest CTA's end time over
    the previous phase's, averaged over layers 1..L-2 of the last of 8 greedy steps - and the
    mean per-CTA time in it.  Not a benchmark value: the trace stores a timestamp per phase."""
    import ctypes

    from dpuf_b200 import engine, model as mdl

    os.environ["DPUF_CUDA_TRACE_DECODE"] = "1"
    shape = model_shape(args.model)
    m = mdl.SyntheticModel(shape, seed=0)
    e = engine.CudaTransformerEngine(m)
    prompt = mdl.prompt_ids(32, shape.vocab, 1)
    e.reset_cache()
    tok = int(np.argmax(e.forward_batch(prompt, 0)[0]))
    for _ in range(max(3, args.warmup)):
        _, ms = e.decode_greedy(tok, len(prompt), 8)
    lib = e.lib
    n_ctas, per = ctypes.c_int32(), ctypes.c_int32()
    lib.dpuf_cuda_decode_trace.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int64]
    lib.dpuf_cuda_decode_trace(e._handle, ctypes.byref(n_ctas), ctypes.byref(per), None, 0)
    C, P = n_ctas.value, per.value
    out = np.zeros(C * P, np.uint64)
    if lib.dpuf_cuda_decode_trace(e._handle, ctypes.byref(n_ctas), ctypes.byref(per), out.ctypes.data, out.size):
        raise RuntimeError("no decode trace (persistent kernel not used?)")
    e.close()
    if args.trace_out:
        np.save(args.trace_out, out.reshape(C, P))
    L = shape.layers
    E = len(TRACE_EVENTS)
    t = out.reshape(C, P).astype(np.int64)
    sb = E * L  # per-step events: start, embedding, final norm, LM head, argmax
    tt = (t - t[:, sb].min()) / 1000.0
    crit, mean = np.zeros(E), np.zeros(E)
    for l in range(1, L - 1):
        prev = tt[:, E * (l - 1) + E - 1]
        for j in range(E):
            cur = tt[:, E * l + j]
            crit[j] += cur.max() - prev.max()
            mean[j] += float(np.mean(cur - prev))
            prev = cur
    crit /= L - 2
    mean /= L - 2
    lm = L // 2
    i_attn, i_qkv = TRACE_EVENTS.index("attn"), TRACE_EVENTS.index("qkv")
    d_attn = tt[:, E * lm + i_attn] - tt[:, E * lm + i_qkv]
    n_attn = int(np.sum(d_attn > 2 * np.median(d_attn) + 1.0))
    print(json.dumps({
        "trace": "decode_kernel phases", "model": shape.name, "ctas": C, "step_us": round(float(tt[:, sb + 4].max()), 1),
        "device_ms_per_step_untraced_run": round(ms / 8, 4),
        "layer_us": round(float(crit.sum()), 2),
        "critical_us": {k: round(float(v), 2) for k, v in zip(TRACE_EVENTS, crit)},
        "mean_cta_us": {k: round(float(v), 2) for k, v in zip(TRACE_EVENTS, mean)},
        "attention_ctas": n_attn, "attention_us_layer_mid": round(float(d_attn.max()), 2),
        "lm_head_us": round(float(tt[:, sb + 3].max() - tt[:, sb + 2].max()), 1),
    }), flush=True)


def profile_value(name: str, key: str):
    """A number recorded in a committed ncu summary under profiles/ (`key: value` line), or None."""
    prof = REPO / "profiles" / name
    if not prof.exists():
        return None
    for line in prof.read_text().splitlines():
        if line.startswith(key + ":"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


def decode_roofline(wbytes: int, step_s: float, hbm_peak: float, peak_kind: str):
    """Roofline of the persistent decode kernel: one launch runs all timed steps, each step
    streams the layer + LM-head weights once (the algorithmic bytes)."""
    ratio = profile_value("decode_kernel_qwen3-8b-l4_step.md", "traffic_per_algorithmic_byte")
    achieved = wbytes / step_s / 1e9
    return {"kernel": "decode_kernel (persistent, one step)", "bound": "hbm", "achieved": round(achieved, 1),
            "peak": hbm_peak, "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
            "traffic": int(wbytes * ratio) if ratio else None, "algorithmic_bytes_per_step": wbytes,
            "us_per_step": round(step_s * 1e6, 2),
            "traffic_note": "dram bytes per algorithmic byte from the ncu capture of the 8B shape cut to 4 layers, "
                            "times the 8B step bytes"}


def prefill_roofline(shape, n_tokens: int, pp_s: float, hbm_peak: float, peak_kind: str) -> dict:
    """Roofline of a host-timed prefill through dpuf_engine_forward_batch (only the last row's
    logits): the tensor-core GEMMs stream each layer matrix's expanded copy once, the LM head
    runs once on the last token (the mode-12 GEMV over its tiles).  The time includes the
    call's copies, the activation preps, attention and norms, so this is a lower bound of the
    GEMMs' own fraction."""
    head = (shape.vocab + 15) // 16 * ((16 + 2 * (shape.hidden // 32) * 144 + 63) // 64 * 64)  # LM-head tiles
    b = shape.layers * shape.expanded_bytes_per_layer() + head
    macs = n_tokens * shape.layers * sum(r * c for _, r, c in shape.linear_shapes()) + shape.vocab * shape.hidden
    return {"bound": "hbm", "bytes": b, "achieved_gbs": round(b / pp_s / 1e9, 1),
            "frac": round(b / pp_s / 1e9 / hbm_peak, 4), "peak": hbm_peak, "peak_kind": peak_kind,
            "int_tops": round(2 * macs / pp_s / 1e12, 2),
            "bytes_what": "expanded copies of every layer matrix (4,352 B per 128 rows x 32 columns) + LM-head tiles",
            "timing": "host clock around one forward_batch call (copies, preps, attention and norms included)"}


MODEL_FORMAT = "v1"  # bump when the synthetic model or the container layout changes


def cache_dir() -> pathlib.Path:
    """Where the benchmark's .dpuf model files live: env DPUF_BENCH_CACHE, else /dev/shm when it
    has room for two 8B models, else .bench_cache/ in the repository."""
    env = os.environ.get("DPUF_BENCH_CACHE")
    if env:
        return pathlib.Path(env)
    try:
        st = os.statvfs("/dev/shm")
        if st.f_bavail * st.f_frsize > 12 * 2**30:
            return pathlib.Path("/dev/shm/dpuf_bench")
    except OSError:
        pass
    return REPO / ".bench_cache"


def model_shape(name: str):
    """--model: "8b" (the benchmark), "0.6b" (configuration 1), "8b-l4" (the 8B shape cut to four
    layers, for profiler captures only)."""
    from dpuf_b200 import model as mdl

    return {"8b": mdl.QWEN3_8B, "0.6b": mdl.QWEN3_0_6B, "8b-l4": mdl.QWEN3_8B_L4}[name]


def model_file(shape_name: str, seed: int = 0) -> pathlib.Path:
    """The random-init model `shape_name` as a DPUF0001 container, written once by a separate
    process (python -m dpuf_b200.container write), so that the process that reads it - the CPU
    reference arm in particular - maps no library of this package."""
    path = cache_dir() / f"{shape_name}-seed{seed}-{MODEL_FORMAT}.dpuf"
    if not path.exists():
        env = dict(os.environ)
        env.pop("OMP_NUM_THREADS", None)
        subprocess.run([sys.executable, "-m", "dpuf_b200.container", "write", str(path), "--shape", shape_name,
                        "--seed", str(seed)], cwd=str(REPO), env=env, check=True, stdout=subprocess.DEVNULL)
    return path


def shared_model_file(shape_name: str, world: int, rank: int) -> pathlib.Path:
    """model_file() made by rank 0 while the other ranks wait at a barrier."""
    if rank == 0:
        path = model_file(shape_name)
    barrier(world)
    if rank != 0:
        path = model_file(shape_name)
    return path


def bench_config(shape, world: int, parallelism: str) -> dict:
    """The `config` object of both arms' lines (same workload, same keys)."""
    return {"workload": f"{shape.name}-shape random-init mode-12 .dpuf, pp32 then batch-1 greedy decode",
            "layers": shape.layers, "hidden": shape.hidden, "vocab": shape.vocab, "prompt": 32,
            "batch": 1, "kv": "fp32", "parallelism": parallelism, "n_gpus": world,
            "l2": f"weights {shape.weight_bytes_per_token() / 1e9:.2f} GB > 126 MB L2: every step streams them from HBM"}


def cpu_threads() -> int:
    """Threads for the reference CPU engine: every core this process may use (the engine caps
    its team at 32, dpuf_engine.c:1220)."""
    from oracle import oracle as orc

    return min(32, orc.host_threads())


def cpu_baseline(m, prompt, n_steps: int, threads: int):
    from oracle import oracle as orc

    if not orc.RefEngine.available():
        return None
    ref = orc.RefEngine(m, n_threads=threads)
    ref.reset()
    t0 = time.perf_counter()
    lg = ref.forward(prompt, 0, 1)[0]
    pp_s = time.perf_counter() - t0
    nxt = int(np.argmax(lg))
    pos = len(prompt)
    t0 = time.perf_counter()
    for _ in range(n_steps):
        lg = ref.forward(np.array([nxt], np.int32), pos, 1)[0]
        nxt = int(np.argmax(lg))
        pos += 1
    dt = time.perf_counter() - t0
    used = ref.threads
    ref.close()
    return {"value": round(n_steps / dt, 3), "unit": "tok/s", "cores": used, "kind": "reference",
            "prefill_tok_per_s": round(len(prompt) / pp_s, 2),
            "sample": f"{n_steps} greedy decode steps after pp{len(prompt)} (prefill_tok_per_s: that one "
                      f"forward_batch call) on the same .dpuf model, reference AVX2/OpenMP engine with {used} "
                      f"OpenMP threads, {orc.cpu_model_string()}"}


def run_reference(args, world, rank):
    """--impl reference: the reference's CPU engine (oracle/_ref/libdpuf_avx2.so, built from its
    unmodified sources) on this host, through its own C ABI, over the same .dpuf file as the
    GPU arm: same workload, metric and config.  This process maps no library of this package:
    the model file is written by a separate process and read here with numpy."""
    from dpuf_b200 import container, model as mdl
    from oracle import oracle as orc

    shape = model_shape(args.model)
    parallelism = ("single" if world == 1 else (f"dp{world}" if args.dp else f"tp{world}"))
    if rank != 0:
        return
    if not orc.RefEngine.available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libdpuf_avx2.so not built "
                                                              "(needs the reference sources at build time)"}))
        return
    m = container.DpufFile(model_file(shape.name))
    threads = cpu_threads()
    prompt = mdl.prompt_ids(32, shape.vocab, 0)
    ref = orc.RefEngine(m, n_threads=threads)
    used = ref.threads
    ref.reset()
    ref.forward(prompt, 0, 1)  # first touch of the mapped weights
    ref.reset()
    t0 = time.perf_counter()
    lg = ref.forward(prompt, 0, 1)[0]
    pp_s = time.perf_counter() - t0
    nxt = int(np.argmax(lg))
    pos = 32
    for _ in range(args.warmup):
        nxt = int(np.argmax(ref.forward(np.array([nxt], np.int32), pos, 1)[0]))
        pos += 1
    t0 = time.perf_counter()
    for _ in range(args.steps):
        nxt = int(np.argmax(ref.forward(np.array([nxt], np.int32), pos, 1)[0]))
        pos += 1
    dt = time.perf_counter() - t0
    ref.close()
    v = args.steps / dt
    print(json.dumps({
        "impl": "reference", "metric": "decode_tok_per_s", "value": round(v, 3), "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "weak" if args.dp else "strong", "vs_baseline": None,
        "dtype": "int8xint4->f32", "data": "synthetic random-init weights ~N(0,0.02), seed-0 prompt",
        "config": bench_config(shape, world, parallelism),
        "prefill": {"tok_per_s": round(32 / pp_s, 3)},
        "cpu_baseline": {"value": round(v, 3), "unit": "tok/s", "cores": used, "kind": "reference",
                         "sample": f"{args.steps} decode steps after pp32, {used} OpenMP threads, "
                                   f"{orc.cpu_model_string()}"},
        "e2e": {"value": round(v, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def greedy_record(eng, prompt, n_logit_steps: int, n_greedy: int):
    """pp(prompt) plus n_logit_steps forward_token steps with host logits (all kept), then
    n_greedy device-fed greedy steps (ids kept): the sequence the parity check compares."""
    eng.reset_cache()
    lg = eng.forward_batch(prompt, 0)[0]
    logits = [lg.copy()]
    nxt, pos = int(np.argmax(lg)), len(prompt)
    ids = [nxt]
    for _ in range(n_logit_steps):
        lg = eng.forward_token(nxt, pos)
        logits.append(lg.copy())
        nxt = int(np.argmax(lg))
        ids.append(nxt)
        pos += 1
    g, _ = eng.decode_greedy(nxt, pos, n_greedy)
    return ids + [int(x) for x in g], np.stack(logits)


def run_dpuf(args, world, rank, local):
    import torch

    from dpuf_b200 import container, engine, model as mdl

    torch.cuda.set_device(local)
    hbm_peak, peak_kind = peaks()
    shape = model_shape(args.model)
    tp = world > 1 and not args.dp
    parallelism = "single" if world == 1 else (f"tp{world}" if tp else f"dp{world}")
    t_build = time.perf_counter()
    m = container.DpufFile(shared_model_file(shape.name, world, rank))
    t_build = time.perf_counter() - t_build
    # data parallel: each rank decodes its own sequence (rank 0 uses the seed-0 prompt); tensor
    # parallel: all ranks decode the seed-0 sequence together
    prompt = mdl.prompt_ids(32, shape.vocab, 0 if tp else rank)
    n_total = args.warmup + args.steps
    if 32 + 2 * n_total + 8 > shape.max_seq:
        raise SystemExit("steps + warmup exceed the 2304-position context")

    # ---- tensor parallel: every rank first records the sequence on its GPU alone (the 1-GPU
    # reference of the parity check), then joins the split engine and records it again
    parity = None
    ids_1 = None
    if tp:
        solo = engine.CudaTransformerEngine(m)
        ids_1, lg_1 = greedy_record(solo, prompt, 4, n_total)
        solo.close()
    eng = engine.CudaTransformerEngine(m)
    lib = eng.lib
    if tp:
        eng.tp_attach(rank, world, engine.torch_all_gather())
        ids_n, lg_n = greedy_record(eng, prompt, 4, n_total)
        parity = ids_n == ids_1 and np.array_equal(lg_n.view(np.uint32), lg_1.view(np.uint32))

    # ---- pp32 (prefill) through the C ABI
    eng.reset_cache()
    eng.forward_batch(prompt, 0)
    eng.reset_cache()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    lg = eng.forward_batch(prompt, 0)[0]
    pp_s = time.perf_counter() - t0
    first = int(np.argmax(lg))

    # ---- device-timed decode (value): W warm-up steps, then K steps in one call
    ids = np.zeros(n_total, np.int32)
    ms = ctypes.c_float()
    rc = lib.dpuf_cuda_decode_greedy(eng._handle, first, 32, args.warmup, ids.ctypes.data, ctypes.byref(ms))
    if rc != 0:
        raise RuntimeError(engine.last_error())
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        rc = lib.dpuf_cuda_decode_greedy(eng._handle, int(ids[args.warmup - 1]), 32 + args.warmup, args.steps,
                                         ids[args.warmup:].ctypes.data, ctypes.byref(ms))
        torch.cuda.synchronize()
    if rc != 0:
        raise RuntimeError(engine.last_error())
    barrier(world)
    if tp:
        value, dev_ms = tp_value(float(ms.value), args.steps, world)
        # the timed run (pp32 id, then device-fed steps from position 32) is the same greedy
        # sequence as the recording (pp32 id, 4 host-logit steps, device-fed steps)
        timed = [first] + [int(x) for x in ids]
        parity = parity_agreed(parity and timed == ids_1[:len(timed)], world)
    else:
        value, dev_ms = dp_value(float(ms.value), args.steps, world)

    if args.no_extras:
        persistent = eng.persistent_decode()[0]
        eng.close()
        if rank == 0:
            print(json.dumps({"metric": "decode_tok_per_s", "value": round(value, 2), "unit": "tok/s",
                              "model": shape.name, "ms_per_step": round(dev_ms / args.steps, 4),
                              "persistent": persistent, "tp_parity": parity}), flush=True)
        return 0 if parity is not False else 1
    # ---- e2e through the drop-in C ABI with host buffers (token id in, logits out)
    eng.reset_cache()
    lg = eng.forward_batch(prompt, 0)[0]
    nxt = int(np.argmax(lg))
    pos = 32
    for _ in range(args.warmup):
        lg = eng.forward_token(nxt, pos)
        nxt = int(np.argmax(lg))
        pos += 1
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        lg = eng.forward_token(nxt, pos)
        nxt = int(np.argmax(lg))
        pos += 1
    e2e_s = allreduce_max(time.perf_counter() - t0, world)
    e2e = (1 if tp else world) * args.steps / e2e_s

    roof = None
    gemv = None
    cpu = None
    persistent, why = eng.persistent_decode()
    wbytes = shape.weight_bytes_per_token()
    if tp:  # each GPU streams its share of the weights
        wbytes //= world
    step_s = dev_ms * 1e-3 / args.steps
    eng.close()
    if rank == 0:
        roof = decode_roofline(wbytes, step_s, hbm_peak, peak_kind) if persistent else None
        gemv = gemv_roofline(hbm_peak, peak_kind)
        if roof is None:
            roof = gemv
        cpu = cpu_baseline(m, prompt, n_steps=24, threads=cpu_threads())
    if rank != 0:
        return 0 if parity is not False else 1
    clocks = clk.summary()
    line = {
        "metric": "decode_tok_per_s", "value": round(value, 2), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 4),
        "higher_is_better": True, "scaling": "weak" if (world > 1 and not tp) else "strong", "vs_baseline": None,
        "dtype": "int8xint4->f32",
        "data": "synthetic random-init weights ~N(0,0.02) (bf16-rounded, mode-12 packed .dpuf), seed-0 prompt",
        "config": bench_config(shape, world, parallelism),
        "tp_parity": parity,
        "step_roofline": {"bytes_per_step_per_gpu": wbytes, "achieved_gbs": round(wbytes / step_s / 1e9, 1),
                          "frac": round(wbytes / step_s / 1e9 / hbm_peak, 4), "peak": hbm_peak,
                          "peak_kind": peak_kind},
        "roofline": roof,
        "gemv_kernel": gemv if roof is not gemv else None,
        "decode_path": "persistent cooperative kernel" if persistent else f"per-step kernels ({why})",
        "prefill": {"tok_per_s": round(32 / pp_s, 1), "what": "pp32 through dpuf_engine_forward_batch",
                    "roofline": prefill_roofline(shape, 32, pp_s, hbm_peak, peak_kind)},
        "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": 4 if persistent else 1040,
                "d2h_bytes_per_step": shape.vocab * 4,
                "what": "dpuf_engine_forward_token per step: token id in, logits D2H, host argmax"},
        "cpu_baseline": cpu,
        "clocks": clocks,
        "gpu_launches": None,
        "model_load_s": round(t_build, 1),
    }
    if tp:
        line["tp_parity_check"] = ("every rank's greedy ids (pp32, 4 host-logit steps, then the device-fed steps "
                                   "incl. the timed ones) and its logits (pp32 and the 4 steps) bit-identical to "
                                   "the same sequence on its GPU alone")
    # the timed decode_greedy call is one launch of the persistent kernel (all steps), or the
    # per-step kernels of every step
    line["gpu_launches"] = 1 if persistent else steps_launch_count(shape) * args.steps
    print(json.dumps(line), flush=True)
    return 0 if parity is not False else 1


def steps_launch_count(shape) -> int:
    """Kernels of one per-step decode step: embed; per layer norm, qkv gemv, qk_post, attention,
    prep, o gemv, norm, gate/up gemv, swiglu_prep, down gemv; final norm, lm gemv, greedy advance."""
    return 1 + 10 * shape.layers + 3


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="dpuf", choices=["dpuf", "reference"])
    ap.add_argument("--model", default="8b", choices=["8b", "0.6b", "8b-l4"],
                    help="8b = the benchmark workload; 0.6b = configuration 1; 8b-l4 = the 8B shape cut to "
                         "four layers, for profiler captures")
    ap.add_argument("--gemv-only", action="store_true",
                    help="only the kernel-only GEMV roofline measurement (for profiling the GEMV)")
    ap.add_argument("--op", action="store_true", help="config 2: isolated mode-12 matmuls at M = 1 and 32")
    ap.add_argument("--zone", action="store_true", help="config 4: Zone-A LM head stress")
    ap.add_argument("--serve", action="store_true", help="config 5: batched serving of independent sequences")
    ap.add_argument("--serve-seqs", type=int, default=64)
    ap.add_argument("--serve-prompt", type=int, default=2048)
    ap.add_argument("--serve-steps", type=int, default=256)
    ap.add_argument("--serve-kv", default="f16", choices=["f16", "f32", "q8"],
                    help="KV cache of the serving run: fp16 (the configuration's), fp32 (the reference's "
                         "kv_type 0) or q8 (the reference's kv_type 1)")
    ap.add_argument("--dp", action="store_true",
                    help="with --gpus N > 1: N independent data-parallel replicas (one sequence each) instead of "
                         "the default tensor parallelism over the N GPUs (one sequence)")
    ap.add_argument("--tp", action="store_true", help="(the default for --gpus N > 1) tensor parallelism")
    ap.add_argument("--trace", action="store_true",
                    help="phase trace of the persistent decode kernel (per-layer critical path), not a benchmark")
    ap.add_argument("--trace-out", default="", help="with --trace: also save the raw [CTA][stamp] array (.npy)")
    ap.add_argument("--no-extras", action="store_true",
                    help="decode timing only (no e2e, roofline or CPU baseline), for profiling runs")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world, rank, local = dist_setup(args.gpus)
    if args.trace:
        import torch

        torch.cuda.set_device(local)
        run_trace(args)
        return
    if args.gemv_only or args.op or args.zone or args.serve:
        import torch

        torch.cuda.set_device(local)
        if args.gemv_only:
            print(json.dumps(gemv_roofline(*peaks())), flush=True)
        if args.op:
            run_op_configs(*peaks())
            run_had_op_configs(*peaks())
        if args.zone:
            run_zone_config(*peaks())
        if args.serve:
            try:
                run_serve_config(args, *peaks(), world=world, rank=rank, local=local)
            finally:
                if world > 1:
                    import torch.distributed as dist

                    dist.destroy_process_group()
        return
    rc = 0
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        else:
            rc = run_dpuf(args, world, rank, local) or 0
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
    if rc:
        sys.exit(rc)


if __name__ == "__main__":
    main()
