#!/usr/bin/env python3
"""Benchmark of the MLA hot path on B200 (BASELINE metric: "MLA decode KV GB/s
(% HBM peak) & prefill TFLOP/s at 1/2/4/8 B200").

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload prefill|prefill_cp|decode_q8|decode_q8_step|decode_long|
                                decode_long_stack|decode_stack|decode_parity]

Default workload: BASELINE config 2 (causal MLA prefill, one sequence of 4096
tokens, H=2048, 16 heads; the configuration the metric's prefill half is quoted
on and the largest that fits one GPU).  The decode half of the metric is
reported in the same JSON line under "decode" (config 1 single-sequence
attend, config 3 Q8 batched attend and full step, config 5 long-context
decode and its 27-layer variant, config 4 27-layer batched decode step; KV
GB/s against measured HBM bandwidth), beside the drop-in decode call.

Multi-GPU (torchrun, one rank per GPU): the prefill headline is the one
config-2 prompt context-parallel over the ranks (zigzag query chunks, one NCCL
all-gather of the compressed rows; strong scaling), with one independent
prompt per rank as a sub-line (weak scaling); batched decode shards sequences
across ranks; the long-context decode splits the KV range across ranks and
merges the (o, lse) partials with the library's peer-store exchange kernel
over NVLink.

Inputs are synthetic, seeded (seed = configuration index), created once on the
device; every timed step is preceded by an untimed 256 MiB write that flushes
L2, and each step is timed with CUDA events on the launching stream; the
reported time is the max over ranks.
"""
from __future__ import annotations

import argparse
import ctypes as C
import datetime
import json
import math
import os
import pathlib
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


# ----------------------------------------------------------------------------- helpers
def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


def prefill_flops(S, H=2048, NH=16, DN=128, DR=64, DV=128, R=512):
    proj = 2 * S * (H * (NH * (DN + DR) + R + DR) + R * NH * (DN + DV) + NH * DV * H)
    attn = S * (S + 1) // 2 * NH * 2 * ((DN + DR) + DV)
    return proj, attn


class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None

    def init(self, torch, backend="nccl"):
        if self.world > 1:
            import torch.distributed as dist
            torch.cuda.set_device(self.local)
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", self.local))
            self.pg = dist
        elif torch.cuda.is_available():
            torch.cuda.set_device(0)

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, torch, v: float) -> float:
        if not self.pg:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def sum(self, torch, v: float) -> float:
        if not self.pg:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.SUM)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.proc = None
        self.gpu = gpu_index
        # the raw samples go to $KVL_BENCH_OUT (default: the system temp directory)
        out = os.environ.get("KVL_BENCH_OUT") or tempfile.gettempdir()
        self.path = pathlib.Path(out) / f"kvl_bench_clocks_rank{gpu_index}.csv"

    def start(self):
        try:
            self.path.parent.mkdir(parents=True, exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "200"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.close()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def timed_steps(torch, dist, step, K, W, flush):
    """W untimed warm-ups, then K steps each timed with CUDA events (L2 flushed
    before every step, outside the timed interval).  Returns max-over-ranks ms."""
    stream = torch.cuda.current_stream()
    for _ in range(W):
        flush()
        step()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    for a, b in ev:
        flush()
        a.record(stream)
        step()
        b.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    total = sum(a.elapsed_time(b) for a, b in ev)
    return dist.max(torch, total)


def profile_read(lib):
    buf = C.create_string_buffer(1 << 16)
    n = lib.kvl_mla_cuda_profile_read(buf, len(buf))
    out = {}
    if n > 0:
        for line in buf.value.decode().splitlines():
            name, ms, cnt = line.split(",")
            out[name] = (float(ms), int(cnt))
    return out


def load_lib():
    import kvl_pkg
    kvl_pkg.load()
    import kvl_b200.kvl_mla as K
    lib = K.load()
    lib.kvl_mla_cuda_profile.argtypes = [C.c_int]
    lib.kvl_mla_cuda_profile.restype = C.c_int
    lib.kvl_mla_cuda_profile_read.argtypes = [C.c_char_p, C.c_size_t]
    lib.kvl_mla_cuda_profile_read.restype = C.c_int
    return K, lib


def dev_bf16(torch, shape, std, gen, device):
    return (torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * std).to(torch.bfloat16)


def device_weights(torch, K, cfg, gen, device, std=0.02):
    H, NH, DN, DR, DV, R = cfg.hidden_size, cfg.num_heads, cfg.qk_nope_dim, cfg.qk_rope_dim, cfg.v_head_dim, \
        cfg.kv_lora_rank
    t = {
        "q_proj": dev_bf16(torch, (NH * (DN + DR), H), std, gen, device),
        "kv_a_proj": dev_bf16(torch, (R + DR, H), std, gen, device),
        "kv_a_norm": torch.ones(R, dtype=torch.bfloat16, device=device),
        "kv_b_proj": dev_bf16(torch, (NH * (DN + DV), R), std, gen, device),
        "o_proj": dev_bf16(torch, (H, NH * DV), std, gen, device),
    }
    w = K.KvlMlaDeviceWeights(*[t[k].data_ptr() for k in ("q_proj", "kv_a_proj", "kv_a_norm", "kv_b_proj",
                                                           "o_proj")])
    return t, w


def replay_as_graph(torch, obj, raw, label, attr="_graph"):
    """Runs raw() (a sequence of library launches on the current stream) as a
    CUDA graph captured on first use (kept in obj.<attr>); every replay launches
    every kernel again.  Falls back to raw() if the capture is refused."""
    if getattr(obj, attr, None) is None:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            raw()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        try:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                raw()
            setattr(obj, attr, g)
        except RuntimeError as e:
            print(f"{label}: CUDA graph capture failed ({e}); launching directly", file=sys.stderr)
            setattr(obj, attr, False)
    if getattr(obj, attr):
        getattr(obj, attr).replay()
    else:
        raw()


# ----------------------------------------------------------------------------- shared inputs
_PREFILL_INPUTS = {}


def prefill_inputs(S=4096):
    """Host inputs of config 2, the same for both arms (synth.py, seed 2): bf16
    bit patterns of [q_proj, kv_a_proj, kv_a_norm, kv_b_proj, o_proj] and of the
    token activations x [S][2048]."""
    if S not in _PREFILL_INPUTS:
        import kvl_pkg
        kvl_pkg.load()
        import kvl_b200.synth as SY
        H, NH, DN, DR, DV, R = 2048, 16, 128, 64, 128, 512
        w = [SY.normal_bf16(2, SY.S_WQ, (NH * (DN + DR), H), 0.02), SY.normal_bf16(2, SY.S_WKVA, (R + DR, H), 0.02),
             SY.f32_to_bf16_bits(np.ones(R, np.float32)), SY.normal_bf16(2, SY.S_WKVB, (NH * (DN + DV), R), 0.02),
             SY.normal_bf16(2, SY.S_WO, (H, NH * DV), 0.02)]
        x = SY.normal_bf16(2, SY.S_X, (S, H), 1.0)
        _PREFILL_INPUTS[S] = (w, x)
    return _PREFILL_INPUTS[S]


def prefill_config(S, theta, world):
    """The `config` of the prefill line, printed identically by both arms."""
    proj, attn = prefill_flops(S)
    return {"workload": f"config 2: causal MLA prefill, 1 sequence x {S} tokens per rank", "seq_len": S,
            "hidden": 2048, "heads": 16, "qk_nope": 128, "qk_rope": 64, "v_head": 128, "kv_lora_rank": 512,
            "rope_theta": theta, "x_dtype": "bf16", "weights": "bf16 ~N(0,0.02), kv_a_norm=1",
            "inputs": "synth.py seed 2 (splitmix64 + Box-Muller), the same values in both arms",
            "flops_per_step_per_rank": proj + attn, "flops_projections": proj, "flops_attention": attn,
            "l2": "flushed (256 MiB write) before every step", "parallelism": f"sequence-sharded x{world}"}


# ----------------------------------------------------------------------------- CPU side (reference)
_REF = {}


def _reference():
    from oracle.oracle import REF_SO, Reference
    if "ref" not in _REF:
        _REF["ref"] = Reference(REF_SO)
    return _REF["ref"]


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_reference_prefill(S, theta=50000.0):
    """Times the reference's own kvl_mla_prefill_bf16 (oracle/_ref, AVX2 + OpenMP)
    on one S-token sequence at the config-2 head shapes, on the inputs the GPU
    arm uses.  Returns (seconds, flops)."""
    from oracle.oracle import cfg_of
    import kvl_b200.synth as SY
    w, xb = prefill_inputs(S)
    if ("x", S) not in _REF:
        _REF[("x", S)] = SY.bf16_bits_to_f32(xb)
    cfg = cfg_of(2048, 16, 128, 64, 128, 512, 1e-5, theta)
    ref = _reference()
    t0 = time.perf_counter()
    ref.prefill(_REF[("x", S)], cfg, w)
    dt = time.perf_counter() - t0
    proj, attn = prefill_flops(S)
    return dt, proj + attn


def cpu_reference_decode(L, nseq, threads, q8=False, theta=50000.0, seed=4):
    """Times the reference's own decode call -- kvl_mla_decode_compressed_bf16,
    or kvl_mla_decode_compressed_q8_bf16 with q8 (src/mla_compressed_state.c:86-161,
    src/mla_compressed_q8_state.c:161-255; oracle/_ref, AVX2 + OpenMP) -- once
    for each of `nseq` sequences of L cached rows (synthetic rows written into
    the state, random config-2-shaped weights), `threads` sequences at a time.
    The call is the whole decode of one token: projections, append and the
    attention over L + 1 rows.  Returns seconds for all calls."""
    from concurrent.futures import ThreadPoolExecutor

    from oracle.oracle import cfg_of
    import kvl_b200.kvl_mla as K
    import kvl_b200.synth as SY
    ref = _reference()
    cfg = cfg_of(2048, 16, 128, 64, 128, 512, 1e-5, theta)
    w = K.random_weights(K.make_config(2048, 16, 128, 64, 128, 512, 1e-5, theta), seed, 0.02)
    xs = SY.bf16_bits_to_f32(SY.normal_bf16(seed, SY.S_X, (nseq, 2048), 1.0))
    if q8:
        rows = (SY.uniform_int8(seed, SY.S_LAT, (L, 512)), SY.uniform_f32(seed, SY.S_SCALE, (L,), 0.001, 0.02),
                SY.normal_bf16(seed, SY.S_ROPE, (L, 64), 1.0))
        call = lambda b: ref.decode_q8_from_rows(xs[b], cfg, w.arrays, *rows)  # noqa: E731
    else:
        kv = SY.bf16_bits_to_f32(SY.normal_bf16(seed, SY.S_LAT, (L, 576), 1.0))
        lat, rope = np.ascontiguousarray(kv[:, :512]), np.ascontiguousarray(kv[:, 512:])
        call = lambda b: ref.decode_from_rows(xs[b], cfg, w.arrays, lat, rope)  # noqa: E731
    t0 = time.perf_counter()
    if threads <= 1:
        for b in range(nseq):
            call(b)
    else:
        with ThreadPoolExecutor(max_workers=threads) as ex:
            list(ex.map(call, range(nseq)))
    return time.perf_counter() - t0


def cpu_port_attend_bf16(L, threads=1):
    """The attend core of the reference decode (src/mla_compressed_state.c:132-148)
    through the C restatement (double accumulation, single-threaded as in the
    reference) over L synthetic rows of one sequence.  Returns seconds."""
    from oracle.oracle import Oracle
    import kvl_b200.synth as SY
    orc = Oracle()
    kv = SY.bf16_bits_to_f32(SY.normal_bf16(5, SY.S_LAT, (L, 576), 1.0))
    lat, rope = np.ascontiguousarray(kv[:, :512]), np.ascontiguousarray(kv[:, 512:])
    q = SY.bf16_bits_to_f32(SY.normal_bf16(5, SY.S_Q, (16, 576), 0.1))
    t0 = time.perf_counter()
    orc.attend_f32(q, lat, rope, 1.0 / math.sqrt(192.0))
    return time.perf_counter() - t0


def cpu_reference_decode_q8(lens, threads):
    """Times the reference's attend work for a Q8 batch.  The reference's public
    kvl_mla_decode_compressed_q8_bf16 call is not attend-only, so the attend core
    (src/mla_compressed_q8_state.c:216-238) is timed through the C restatement,
    one worker thread per sequence.  Returns (seconds, bytes)."""
    from concurrent.futures import ThreadPoolExecutor

    from oracle.oracle import Oracle
    import kvl_b200.synth as SY
    orc = Oracle()
    R, DR, NH = 512, 64, 16
    jobs = []
    for b, L in enumerate(lens):
        lat8 = SY.uniform_int8(100 + b, SY.S_LAT, (L, R))
        sc = SY.uniform_f32(100 + b, SY.S_SCALE, (L,), 0.001, 0.02)
        rp = SY.normal_bf16(100 + b, SY.S_ROPE, (L, DR))
        q = SY.bf16_bits_to_f32(SY.normal_bf16(100 + b, SY.S_Q, (NH, R + DR), 0.1))
        jobs.append((q, lat8, sc, rp))
    t0 = time.perf_counter()
    with ThreadPoolExecutor(max_workers=threads) as ex:
        list(ex.map(lambda j: orc.attend_q8(j[0], j[1], j[2], j[3], 1.0 / math.sqrt(192.0)), jobs))
    return time.perf_counter() - t0, sum(lens) * 644


def _cpu_guard(fn):
    try:
        return fn()
    except Exception as e:  # noqa: BLE001 - report, keep the GPU numbers
        return {"error": str(e)}


def decode_cpu_baseline(name, wl):
    """CPU figures of one decode sub-line, on this host's cores.  `cpu_baseline`
    is the reference's own decode call where the line's workload allows it,
    else the C restatement of the reference attend core (kind "port"); each
    says what its sample was."""
    cores = host_threads()
    if name == "decode_parity":
        def run():
            reps = 5
            dt = cpu_reference_decode(wl.L, reps, 1) / reps
            port = cpu_port_attend_bf16(wl.L)
            return {"value": wl.L * 1152 / dt / 1e9, "unit": "GB/s", "cores": cores, "kind": "reference",
                    "sample": f"reference kvl_mla_decode_compressed_bf16 (AVX2 + OpenMP matvecs, serial attention) "
                              f"at L={wl.L}, one call = the whole decode of a token (projections, append, "
                              f"attention), {1e3 * dt:.1f} ms per call (mean of {reps}); KV bytes counted at "
                              "1152 B per row as on the GPU line",
                    "attend_core_port": {"value": wl.L * 1152 / port / 1e9, "unit": "GB/s", "cores": 1,
                                         "sample": f"C restatement of src/mla_compressed_state.c:132-148 over "
                                                   f"{wl.L} rows, {1e3 * port:.2f} ms"}}
        return _cpu_guard(run)
    if name == "decode_long":
        def run():
            n = 16384
            dt = cpu_port_attend_bf16(n)
            return {"value": n * 1152 / dt / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
                    "sample": f"C restatement of the reference attend core (src/mla_compressed_state.c:132-148, "
                              f"single-threaded as the reference) over the first {n} of {wl.L} rows, "
                              f"{dt:.2f} s; the rate is per row, so the whole sequence takes about "
                              f"{dt * wl.L / n:.1f} s (extrapolated)"}
        return _cpu_guard(run)
    if name == "decode_stack":
        def run():
            nseq, thr = 8, min(8, cores)
            dt = cpu_reference_decode(wl.L, nseq, thr)
            nbytes = nseq * wl.L * 1152
            step = dt * wl.LAYERS * (256 / nseq)
            return {"value": nbytes / dt / 1e9, "unit": "GB/s", "cores": thr, "kind": "reference",
                    "sample": f"subset: 1 layer x {nseq} sequences at L={wl.L} through the reference "
                              f"kvl_mla_decode_compressed_bf16 (whole decode call), {thr} sequences in parallel, "
                              f"{dt:.2f} s", "extrapolated": True,
                    "extrapolated_step_s": step,
                    "extrapolation": f"linear: x{wl.LAYERS} layers x {256 // nseq} sequence groups"}
        return _cpu_guard(run)
    if name == "decode_q8_step":
        def run():
            sub = sorted(wl.lens)[len(wl.lens) // 2:len(wl.lens) // 2 + 8]
            thr = min(8, cores)
            t0 = time.perf_counter()
            from concurrent.futures import ThreadPoolExecutor
            with ThreadPoolExecutor(max_workers=thr) as ex:
                list(ex.map(lambda L: cpu_reference_decode(L, 1, 1, q8=True), sub))
            wall = time.perf_counter() - t0
            nbytes = sum(L + 1 for L in sub) * 644
            return {"value": nbytes / wall / 1e9, "unit": "GB/s", "cores": thr, "kind": "reference",
                    "sample": f"subset: 8 of the 64 config-3 sequences ({sum(sub)} rows) through the reference "
                              f"kvl_mla_decode_compressed_q8_bf16 (the whole step of a token: projections, "
                              f"quantised append, attention), {thr} in parallel, {wall:.2f} s wall",
                    "extrapolated": True, "extrapolated_step_s": wall * len(wl.lens) / len(sub),
                    "extrapolation": f"linear: x{len(wl.lens) // len(sub)} sequence groups"}
        return _cpu_guard(run)
    if name == "decode_long_stack":
        def run():
            dt = cpu_reference_decode(wl.L, 1, 1)
            return {"value": wl.L * 1152 / dt / 1e9, "unit": "GB/s", "cores": cores, "kind": "reference",
                    "sample": f"subset: 1 layer of the 27 through the reference kvl_mla_decode_compressed_bf16 "
                              f"(whole decode call: projections, append, serial attention over {wl.L + 1} rows), "
                              f"{dt:.2f} s", "extrapolated": True, "extrapolated_step_s": dt * wl.LAYERS,
                    "extrapolation": f"linear: x{wl.LAYERS} layers"}
        return _cpu_guard(run)
    if name == "decode_q8":
        def run():
            secs, nbytes = cpu_reference_decode_q8(wl.lens, cores)
            res = {"value": nbytes / secs / 1e9, "unit": "GB/s", "cores": cores, "kind": "port",
                   "sample": f"all {len(wl.lens)} sequences ({sum(wl.lens)} rows) of the config-3 attend through the "
                             "C restatement of src/mla_compressed_q8_state.c:216-238 (double accumulation, as the "
                             f"reference), one sequence per thread, {secs:.2f} s"}
            sub = sorted(wl.lens)[len(wl.lens) // 2:len(wl.lens) // 2 + 8]
            thr = min(8, cores)
            t0 = time.perf_counter()
            from concurrent.futures import ThreadPoolExecutor
            with ThreadPoolExecutor(max_workers=thr) as ex:
                times = list(ex.map(lambda L: cpu_reference_decode(L, 1, 1, q8=True), sub))
            wall = time.perf_counter() - t0
            res["reference_call"] = {
                "value": sum(sub) * 644 / wall / 1e9, "unit": "GB/s", "cores": thr, "kind": "reference",
                "sample": f"subset: 8 of the 64 config-3 lengths ({sum(sub)} rows) through the reference "
                          f"kvl_mla_decode_compressed_q8_bf16 (whole decode call per sequence), {thr} in parallel, "
                          f"{wall:.2f} s wall ({1e3 * sum(times) / len(times):.0f} ms per call)"}
            return res
        return _cpu_guard(run)
    return None


# ----------------------------------------------------------------------------- workloads
class Prefill:
    """one 4096-token causal MLA prefill.  On one GPU the
    whole prompt; under torchrun (N > 1) the same prompt context-parallel over
    the N GPUs (mode "cp": zigzag query chunks, one NCCL all-gather of the
    compressed rows between kvl_mla_prefill_cp_begin and _end; strong scaling),
    or one independent prompt per GPU (mode "independent"; weak scaling)."""
    name = "prefill"
    metric = "MLA prefill TFLOP/s (config 2: S=4096, H=2048, 16 heads, causal)"
    unit = "TFLOP/s"
    bound = "tensor"
    # dram__bytes_read.sum + dram__bytes_write.sum per launch, one ncu capture
    # (profiles/flash_prefill_config2.txt, profiles/gemm_prefill_config2.txt)
    ncu_traffic = {"flash_prefill": 59.550720e6 + 3.057408e6, "gemm_q": 30.439168e6 + 0.093440e6}

    def __init__(self, torch, K, lib, dist, S=4096, theta=50000.0, mode=None):
        self.torch, self.K, self.lib, self.dist = torch, K, lib, dist
        self.S = S
        self.mode = mode or ("cp" if dist.world > 1 else "single")
        self.scaling = "strong" if self.mode == "cp" else "weak"
        if self.mode == "independent":
            self.name = "prefill_independent"
        dev = torch.device("cuda", torch.cuda.current_device())
        self.cfg = K.make_config(2048, 16, 128, 64, 128, 512, 1e-5, theta)
        # the same synthetic inputs as the reference arm (synth.py, seed 2)
        w_host, x_host = prefill_inputs(S)
        names = ("q_proj", "kv_a_proj", "kv_a_norm", "kv_b_proj", "o_proj")
        self.w_host = w_host
        self.wt = {k: torch.from_numpy(a.view(np.int16)).to(dev).view(torch.bfloat16) for k, a in zip(names, w_host)}
        self.w = K.KvlMlaDeviceWeights(*[self.wt[k].data_ptr() for k in names])
        self.x = torch.from_numpy(x_host.view(np.int16)).to(dev).view(torch.bfloat16)
        self.out = torch.empty((S, 2048), dtype=torch.float32, device=dev)
        nbytes = lib.kvl_mla_prefill_workspace_bytes(C.byref(self.cfg), S)
        self.ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        self.proj, self.attn = prefill_flops(S)
        self.units = self.proj + self.attn
        if self.mode == "cp":
            import kvl_b200.parallel as PAR
            c = S // (2 * dist.world)
            self.c = c
            # the rank holds only its own rows: early chunk, then late chunk
            self.rows = PAR.rank_rows(S, dist.world, dist.rank)
            self.xr = self.x[torch.from_numpy(self.rows).to(dev)].contiguous()
            self.out = torch.empty((2 * c, 2048), dtype=torch.float32, device=dev)
            # bf16 rows (NCCL has no 16-bit integer type)
            self.send = torch.empty((2 * c, 576), dtype=torch.bfloat16, device=dev)
            self.recv = torch.empty((dist.world * 2 * c, 576), dtype=torch.bfloat16, device=dev)

    def kernel_flops(self):
        """Algorithmic FLOPs per step of each library kernel of the prefill path
        (on this rank: in context-parallel mode its 2c query rows and the keys
        its chunks see; the zigzag split gives every rank 1/N of the causal
        pairs)."""
        S, H, NH, QD, DV, R, DR = self.S, 2048, 16, 192, 128, 512, 64
        if self.mode == "cp":
            rows, world = 2 * self.c, self.dist.world
            kmax = (2 * world - self.dist.rank) * self.c
            return {"flash_prefill": float(self.attn) / world, "gemm_q": 2.0 * rows * H * NH * QD,
                    "gemm_kva": 2.0 * rows * H * (R + DR), "gemm_kvb": 2.0 * kmax * R * NH * (128 + DV),
                    "gemm_o": 2.0 * rows * NH * DV * H}
        return {"gemv_bf16": 2.0 * S * (H * (NH * QD + R + DR) + NH * DV * H),
                "vup": 2.0 * S * NH * DV * R, "absorb": 2.0 * S * NH * 128 * R,
                "mla_attend_bf16": float(self.attn), "flash_prefill": float(self.attn),
                "gemm_q": 2.0 * S * H * NH * QD, "gemm_kva": 2.0 * S * H * (R + DR),
                "gemm_kvb": 2.0 * S * R * NH * (128 + DV), "gemm_o": 2.0 * S * NH * DV * H}

    def _cp_begin(self):
        s = self.torch.cuda.current_stream().cuda_stream
        rc = self.lib.kvl_mla_prefill_cp_begin(C.byref(self.cfg), C.byref(self.w), self.xr.data_ptr(), self.S,
                                               self.dist.rank, self.dist.world, self.send.data_ptr(),
                                               self.ws.data_ptr(), self.ws.numel(), s)
        if rc != 0:
            raise RuntimeError(self.K.last_error())

    def _gather(self):
        """The all-gather of the compressed rows (NCCL; a copy on one rank)."""
        if self.dist.pg:
            self.dist.pg.all_gather_into_tensor(self.recv, self.send)
        else:
            self.recv.copy_(self.send)

    def _cp_end(self):
        s = self.torch.cuda.current_stream().cuda_stream
        rc = self.lib.kvl_mla_prefill_cp_end(C.byref(self.cfg), C.byref(self.w), self.out.data_ptr(), self.S,
                                             self.dist.rank, self.dist.world, self.recv.data_ptr(),
                                             self.ws.data_ptr(), self.ws.numel(), s)
        if rc != 0:
            raise RuntimeError(self.K.last_error())

    def step_profiled(self):
        """The launches of one step issued directly (per-kernel CUDA events)."""
        if self.mode == "cp":
            self._cp_begin()
            self._gather()
            self._cp_end()
            return
        s = self.torch.cuda.current_stream().cuda_stream
        rc = self.lib.kvl_mla_prefill_dev(C.byref(self.cfg), C.byref(self.w), self.out.data_ptr(),
                                          self.x.data_ptr(), self.S, self.ws.data_ptr(), self.ws.numel(), s)
        if rc != 0:
            raise RuntimeError(self.K.last_error())

    def step(self):
        """The same launches replayed as CUDA graphs (both streams of the fork);
        in context-parallel mode the two halves are graphs and the NCCL
        all-gather between them is issued directly."""
        if self.mode == "cp":
            replay_as_graph(self.torch, self, self._cp_begin, "prefill cp begin", "_graph_begin")
            self._gather()
            replay_as_graph(self.torch, self, self._cp_end, "prefill cp end", "_graph_end")
            return
        replay_as_graph(self.torch, self, self.step_profiled, "prefill")

    def value(self, ms_per_step):
        prompts = 1 if self.mode == "cp" else self.dist.world
        return prompts * self.units / (ms_per_step * 1e-3) / 1e12

    def e2e(self, K_steps, W_steps):
        """Public host API kvl_mla_prefill_bf16 with host fp32 activations (weights
        cached on the device, as with a full trunk cache).  In context-parallel
        mode: each rank copies its chunks' rows of the prompt (pinned fp32) to
        the device, rounds them to bf16, runs kvl_mla_prefill_cp_begin, the
        all-gather and kvl_mla_prefill_cp_end, and copies its rows of the output
        back."""
        if self.mode == "cp":
            return self._e2e_cp(K_steps, W_steps)
        torch, K, lib = self.torch, self.K, self.lib
        lib.kvl_mla_cuda_weight_cache(1)
        hw = K.Weights(*self.w_host)
        x = self.x.float().cpu().numpy()
        x_pinned = torch.from_numpy(x).pin_memory().numpy()
        out = torch.empty((self.S, 2048), dtype=torch.float32).pin_memory().numpy()

        def call():
            rc = lib.kvl_mla_prefill_bf16(K.ptr(out, K.f32p), K.ptr(x_pinned, K.f32p), self.S, C.byref(self.cfg),
                                          C.byref(hw.c))
            if rc != 0:
                raise RuntimeError(K.last_error())
        for _ in range(W_steps):
            call()
        self.dist.barrier()
        t0 = time.perf_counter()
        for _ in range(K_steps):
            call()
        dt = (time.perf_counter() - t0) * 1e3 / K_steps
        dt = self.dist.max(torch, dt)
        # The same call with the runtime's own kind of buffers: x and out in
        # pageable (malloc'd) memory and the layer's weights uploaded on every
        # call (no trunk cache).
        x_page = np.array(x, copy=True)
        out_page = np.empty_like(out)
        wbytes = int(sum(a.nbytes for a in self.w_host))
        lib.kvl_mla_cuda_weight_cache(0)
        try:
            def call_page():
                rc = lib.kvl_mla_prefill_bf16(K.ptr(out_page, K.f32p), K.ptr(x_page, K.f32p), self.S,
                                              C.byref(self.cfg), C.byref(hw.c))
                if rc != 0:
                    raise RuntimeError(K.last_error())
            for _ in range(min(W_steps, 2)):
                call_page()
            self.dist.barrier()
            t0 = time.perf_counter()
            for _ in range(K_steps):
                call_page()
            dtp = self.dist.max(torch, (time.perf_counter() - t0) * 1e3 / K_steps)
        finally:
            lib.kvl_mla_cuda_weight_cache(1)
        return {"value": self.value(dt), "unit": self.unit, "ms_per_step": dt,
                "h2d_bytes_per_step": int(x.nbytes), "d2h_bytes_per_step": int(out.nbytes),
                "path": "kvl_mla_prefill_bf16 (host fp32 in/out)",
                "pageable_uncached": {"value": self.value(dtp), "unit": self.unit, "ms_per_step": dtp,
                                      "h2d_bytes_per_step": int(x.nbytes) + wbytes,
                                      "d2h_bytes_per_step": int(out.nbytes),
                                      "path": "kvl_mla_prefill_bf16, x and out in pageable host memory, the "
                                              "layer's weights uploaded on every call (no weight cache)"}}

    def _e2e_cp(self, K_steps, W_steps):
        import kvl_b200.parallel as PAR
        torch, lib = self.torch, self.lib
        (a0, a1), (b0, b1) = PAR.zigzag_chunks(self.S, self.dist.world)[self.dist.rank]
        c = self.c
        x_host = torch.from_numpy(self.x.float().cpu().numpy()).pin_memory()
        out_host = torch.empty((self.S, 2048), dtype=torch.float32).pin_memory()
        xf = torch.empty((2 * c, 2048), dtype=torch.float32, device=self.x.device)
        xb16 = self.xr.view(torch.int16)
        stream = torch.cuda.current_stream()

        def call():
            xf[:c].copy_(x_host[a0:a1], non_blocking=True)
            xf[c:].copy_(x_host[b0:b1], non_blocking=True)
            rc = lib.kvl_mla_bf16_rne(xb16.data_ptr(), xf.data_ptr(), 2 * c * 2048, stream.cuda_stream)
            if rc != 0:
                raise RuntimeError(self.K.last_error())
            self._cp_begin()
            self._gather()
            self._cp_end()
            out_host[a0:a1].copy_(self.out[:c], non_blocking=True)
            out_host[b0:b1].copy_(self.out[c:], non_blocking=True)
            stream.synchronize()
        for _ in range(W_steps):
            call()
        self.dist.barrier()
        t0 = time.perf_counter()
        for _ in range(K_steps):
            call()
        dt = (time.perf_counter() - t0) * 1e3 / K_steps
        dt = self.dist.max(torch, dt)
        rows = (a1 - a0) + (b1 - b0)
        return {"value": self.value(dt), "unit": self.unit, "ms_per_step": dt,
                "h2d_bytes_per_step": int(rows * 2048 * 4 * self.dist.world),
                "d2h_bytes_per_step": int(rows * 2048 * 4 * self.dist.world),
                "path": "per rank: its chunks' rows (pinned fp32) -> device, kvl_mla_bf16_rne, kvl_mla_prefill_cp_begin, "
                        "NCCL all-gather, kvl_mla_prefill_cp_end, its rows of the output -> host; bytes summed "
                        "over ranks"}

    def config(self):
        cfg = prefill_config(self.S, self.cfg.rope_theta, self.dist.world)
        if self.mode == "cp":
            cfg["parallelism"] = (f"context-parallel x{self.dist.world}: zigzag query chunks of {self.c} rows, one "
                                  "NCCL all-gather of the compressed 576-wide rows per step")
            cfg["workload"] = f"config 2: causal MLA prefill, 1 sequence x {self.S} tokens over all ranks"
        return cfg

    def launch(self):
        if self.mode == "cp":
            return "kvl_mla_prefill_cp_begin / _end as two CUDA graphs with the NCCL all-gather issued between them"
        return ("kvl_mla_prefill_dev captured once as a CUDA graph (both streams), replayed per step"
                if getattr(self, "_graph", None) else "kvl_mla_prefill_dev launched per step")

    def cpu_baseline(self):
        cores = int(os.environ.get("OMP_NUM_THREADS", host_threads()))
        dt, fl = cpu_reference_prefill(self.S)
        return {"value": fl / dt / 1e12, "unit": self.unit, "cores": cores, "kind": "reference",
                "sample": f"one full config-2 step: reference kvl_mla_prefill_bf16 (AVX2+OpenMP, oracle/_ref) on "
                          f"one {self.S}-token sequence ({fl / 1e9:.2f} GFLOP, {dt:.2f} s)"}


class DecodeQ8:
    """64 sequences, ragged L ~ U[512, 8192], Q8 latent."""
    name = "decode_q8"
    metric = "MLA Q8 decode KV GB/s (config 3: 64 seqs, L~U[512,8192])"
    unit = "GB/s"
    bound = "hbm"
    # the attend's arithmetic: int8 rows x int8 query / softmax-weight parts on
    # the tensor cores with int32 sums, the rope term bf16 with fp32 sums
    dtype = "s8 (int32 accumulate; rope bf16)"
    # one ncu capture of the attend kernel (profiles/mla_attend_q8_config3.txt)
    ncu_traffic = {"mla_attend_q8": 192.881408e6 + 4.977152e6}

    def __init__(self, torch, K, lib, dist):
        import kvl_b200.synth as SY
        import kvl_b200.parallel as PAR
        self.torch, self.K, self.lib, self.dist = torch, K, lib, dist
        lens_all = [int(v) for v in SY.uniform_ints(3, SY.S_LEN, 64, 512, 8192)]
        mine = PAR.shard_sequences(lens_all, dist.world)[dist.rank]
        self.lens = [lens_all[i] for i in mine]
        self.total_bytes = sum(lens_all) * 644
        rows = sum(self.lens)
        row0 = np.concatenate([[0], np.cumsum(self.lens)[:-1]]).astype(np.int64)
        dev = torch.device("cuda", torch.cuda.current_device())
        g = torch.Generator(device=dev)
        g.manual_seed(3 + 1000 * dist.rank)
        self.lat8 = torch.randint(-127, 128, (rows, 512), generator=g, device=dev, dtype=torch.int8)
        self.scale = torch.rand((rows,), generator=g, device=dev) * 0.019 + 0.001
        self.rope = dev_bf16(torch, (rows, 64), 1.0, g, dev)
        self.q = dev_bf16(torch, (len(self.lens), 16, 576), 0.1, g, dev).float()
        self.out = torch.empty((len(self.lens), 16, 512), device=dev)
        self.plan = K.AttendPlan(self.lens, row0, 16, 512)
        self.rows = rows
        self.units = rows * 644

    def step(self):
        s = self.torch.cuda.current_stream().cuda_stream
        rc = self.plan.attend_q8(self.out, None, self.q, self.lat8, self.scale, self.rope, self.rows, stream=s)
        if rc != 0:
            raise RuntimeError(self.K.last_error())

    def value(self, ms):
        return self.total_bytes / (ms * 1e-3) / 1e9

    def e2e_io(self):
        """Per step: the absorbed queries in, the latent contexts out."""
        return [self.q], [self.out]

    def config(self):
        return {"workload": "config 3: Q8 batched decode attend, 64 seqs", "lens_sum": int(sum(self.lens)),
                "bytes_per_token": 644, "parallelism": f"sequence-sharded x{self.dist.world}"}


class DecodeQ8Step:
    """BASELINE config 3 as a full decode step: for the 64 Q8 sequences, one
    kvl_mla_decode_step_q8 (q/kv_a projections, the reference row quantiser
    appending each token's row, the int8 attend over L + 1 rows, V
    up-projection and o_proj) on random config-2-shaped weights; the
    batched form of src/mla_compressed_q8_state.c:161-255."""
    name = "decode_q8_step"
    metric = "MLA Q8 decode step KV GB/s (config 3 full step: 64 seqs, L~U[512,8192])"
    unit = "GB/s"
    bound = "hbm"
    dtype = DecodeQ8.dtype

    def __init__(self, torch, K, lib, dist):
        import kvl_b200.synth as SY
        import kvl_b200.parallel as PAR
        self.torch, self.K, self.lib, self.dist = torch, K, lib, dist
        lens_all = [int(v) for v in SY.uniform_ints(3, SY.S_LEN, 64, 512, 8192)]
        mine = PAR.shard_sequences(lens_all, dist.world)[dist.rank]
        self.lens = [lens_all[i] for i in mine]
        self.total_bytes = sum(L + 1 for L in lens_all) * 644
        rows_seq = [L + 1 for L in self.lens]
        self.rows = sum(rows_seq)
        row0 = np.concatenate([[0], np.cumsum(rows_seq)[:-1]]).astype(np.int64)
        dev = torch.device("cuda", torch.cuda.current_device())
        g = torch.Generator(device=dev)
        g.manual_seed(33 + 1000 * dist.rank)
        self.lat8 = torch.randint(-127, 128, (self.rows, 512), generator=g, device=dev, dtype=torch.int8)
        self.scale = torch.rand((self.rows,), generator=g, device=dev) * 0.019 + 0.001
        self.rope = dev_bf16(torch, (self.rows, 64), 1.0, g, dev)
        self.cfg = K.make_config(2048, 16, 128, 64, 128, 512, 1e-5, 50000.0)
        self.wt, self.w = device_weights(torch, K, self.cfg, g, dev)
        self.n = len(self.lens)
        self.x = dev_bf16(torch, (self.n, 2048), 1.0, g, dev).float()
        self.out = torch.empty((self.n, 2048), dtype=torch.float32, device=dev)
        self.plan = K.AttendPlan(rows_seq, row0, 16, 512)
        self.d_row = torch.from_numpy(row0 + np.array(self.lens, np.int64)).to(dev)
        self.d_pos = torch.tensor(self.lens, dtype=torch.int32, device=dev)
        nbytes = lib.kvl_mla_decode_step_workspace_bytes(C.byref(self.cfg), self.n)
        self.ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        self.units = self.rows * 644

    def step_profiled(self):
        s = self.torch.cuda.current_stream().cuda_stream
        rc = self.lib.kvl_mla_decode_step_q8(
            C.byref(self.cfg), C.byref(self.w), self.plan.h, self.out.data_ptr(), self.x.data_ptr(),
            self.lat8.data_ptr(), self.scale.data_ptr(), self.rope.data_ptr(), self.rows, self.d_row.data_ptr(),
            self.d_pos.data_ptr(), self.n, self.ws.data_ptr(), s)
        if rc != 0:
            raise RuntimeError(self.K.last_error())

    def step(self):
        """The step's launches captured once as a CUDA graph, replayed per step
        (each replay appends at the same rows, as a re-run of the same token)."""
        replay_as_graph(self.torch, self, self.step_profiled, "decode_q8_step")

    def e2e_io(self):
        """Per step: the tokens' hidden states in, the layer outputs out."""
        return [self.x], [self.out]

    def value(self, ms):
        return self.total_bytes / (ms * 1e-3) / 1e9

    def config(self):
        return {"workload": "config 3 as a full Q8 decode step (one layer), 64 seqs", "lens_sum": int(sum(self.lens)),
                "bytes_per_token": 644, "weights": "bf16 ~N(0,0.02), read once per step (27.5 MB, not counted)",
                "launch": ("the step captured once as a CUDA graph, replayed per step"
                           if getattr(self, "_graph", None) else "launched per step"),
                "parallelism": f"sequence-sharded x{self.dist.world}"}


class DecodeLong:
    """one sequence at 131072 cached tokens (bf16 latent),
    split-KV across ranks with an (o, lse) merge over NCCL."""
    name = "decode_long"
    metric = "MLA long-context decode KV GB/s (config 5: L=131072)"
    unit = "GB/s"
    bound = "hbm"
    # one ncu capture of the attend kernel at world size 1 (profiles/mla_attend_bf16_config5.txt)
    ncu_traffic = {"mla_attend_bf16": 151.122944e6 + 4.220672e6}

    def __init__(self, torch, K, lib, dist, L=131072):
        self.torch, self.K, self.lib, self.dist = torch, K, lib, dist
        self.L = L
        per = (L + dist.world - 1) // dist.world
        lo = min(L, dist.rank * per)
        hi = min(L, lo + per)
        self.n = hi - lo
        dev = torch.device("cuda", torch.cuda.current_device())
        g = torch.Generator(device=dev)
        g.manual_seed(5)
        self.kv = dev_bf16(torch, (max(self.n, 1), 576), 1.0, g, dev)
        gq = torch.Generator(device=dev)
        gq.manual_seed(55)
        self.q = dev_bf16(torch, (1, 16, 576), 0.1, gq, dev).float()
        # this rank's (o, lse) as one packed record [16][512] ++ [16], so one
        # all-gather moves both
        self.rec = torch.empty((16 * 512 + 16,), device=dev)
        self.o = self.rec[:16 * 512].view(1, 16, 512)
        self.lse = self.rec[16 * 512:].view(1, 16)
        self.plan = K.AttendPlan([self.n], [0], 16, 512)
        self.peer = None
        if dist.world > 1:
            self.grec = torch.empty((dist.world, 16 * 512 + 16), device=dev)
            self.final = torch.empty((1, 16, 512), device=dev)
            self.final_lse = torch.empty((1, 16), device=dev)
            # the records cross NVLink by peer stores inside one merge kernel;
            # NCCL all-gather + merge where CUDA IPC is not available
            ok = 1.0
            try:
                def gather(b):
                    lst = [None] * dist.world
                    dist.pg.all_gather_object(lst, b)
                    return lst
                self.peer = K.PeerGroup(dist.rank, dist.world, 1, gather)
            except Exception as e:  # noqa: BLE001
                print(f"decode_long: peer exchange unavailable ({e}); using NCCL", file=sys.stderr)
                ok = 0.0
            if dist.sum(torch, ok) < dist.world:  # every rank takes the same path
                if self.peer is not None:
                    self.peer.close()
                self.peer = None
        self.units = self.n * 1152
        self.total_bytes = L * 1152

    def step(self):
        torch = self.torch
        s = torch.cuda.current_stream().cuda_stream
        if self.peer is not None:
            # attend, then one kernel: local combine, peer stores, cross-GPU merge
            rc = self.peer.attend_exchange(self.plan, self.final, self.final_lse, self.q, self.kv, self.n, stream=s)
            if rc != 0:
                raise RuntimeError(self.K.last_error())
            return
        rc = self.plan.attend_bf16(self.o, self.lse, self.q, self.kv, self.n, stream=s)
        if rc != 0:
            raise RuntimeError(self.K.last_error())
        if self.dist.world > 1:
            self.dist.pg.all_gather_into_tensor(self.grec, self.rec)
            rc = self.lib.kvl_mla_merge_packed(self.final.data_ptr(), self.final_lse.data_ptr(), self.grec.data_ptr(),
                                               self.dist.world, 1, 16, 512, s)
            if rc != 0:
                raise RuntimeError(self.K.last_error())

    def value(self, ms):
        return self.total_bytes / (ms * 1e-3) / 1e9

    def e2e_io(self):
        """Per step: the absorbed query in, the merged (o, lse) out."""
        return [self.q], [self.final if self.dist.world > 1 else self.rec]

    def config(self):
        if self.dist.world == 1:
            par = "one GPU: attend + local combine"
        elif self.peer is not None:
            par = (f"split-KV x{self.dist.world} + local combine, peer-store exchange and merge in one kernel "
                   "after the attend (NVLink)")
        else:
            par = f"split-KV x{self.dist.world} + one NCCL all-gather of packed (o, lse) + merge"
        return {"workload": "config 5: long-context decode attend, L=131072", "rows_per_rank": self.n,
                "parallelism": par}


class DecodeStack:
    """one decode step of the 27-layer text stack for 256
    sequences at 32768 cached tokens each (bf16 latent pools), every layer a full
    kvl_mla_decode_step_bf16 (projections, append of the new row, attend over
    32769 rows, V up-projection, o_proj).  Sequences are sharded across ranks
    (equal lengths, so each rank owns 256/N).  27 layers of KV (260.9 GB) do not
    fit one GPU: below 27 x per-layer bytes of free memory the layers cycle
    through `nbuf` distinct pools (each far larger than L2), so every layer still
    reads its full KV bytes from HBM."""
    name = "decode_stack"
    metric = "MLA 27-layer decode KV GB/s (config 4: 256 seqs x 32768)"
    unit = "GB/s"
    bound = "hbm"
    LAYERS = 27

    def __init__(self, torch, K, lib, dist, seqs=256, L=32768, mem_frac=0.85, max_pools=27):
        import kvl_b200.parallel as PAR
        self.torch, self.K, self.lib, self.dist = torch, K, lib, dist
        self.L = L
        mine = PAR.shard_sequences([L] * seqs, dist.world)[dist.rank]
        self.n = len(mine)
        rows_seq = L + 1  # cached rows + the row this step appends
        self.rows = self.n * rows_seq
        dev = torch.device("cuda", torch.cuda.current_device())
        layer_bytes = self.rows * 1152
        free, _ = torch.cuda.mem_get_info(dev)
        self.nbuf = int(max(1, min(self.LAYERS, max_pools, (free * mem_frac) // layer_bytes)))
        if self.nbuf < min(4, self.LAYERS):
            raise RuntimeError(f"config 4 needs 4 layer pools of {layer_bytes / 1e9:.1f} GB; "
                               f"{free / 1e9:.1f} GB free")
        g = torch.Generator(device=dev)
        g.manual_seed(4 + 1000 * dist.rank)
        self.kv = [torch.randn((self.rows, 576), generator=g, device=dev, dtype=torch.bfloat16)
                   for _ in range(self.nbuf)]
        self.cfg = K.make_config(2048, 16, 128, 64, 128, 512, 1e-5, 50000.0)
        self.wt, self.w = [], []
        for _ in range(self.LAYERS):
            t, w = device_weights(torch, K, self.cfg, g, dev)
            self.wt.append(t)
            self.w.append(w)
        self.x = [dev_bf16(torch, (self.n, 2048), 1.0, g, dev).float() for _ in range(self.LAYERS)]
        self.out = torch.empty((self.LAYERS, self.n, 2048), dtype=torch.float32, device=dev)
        row0 = np.arange(self.n, dtype=np.int64) * rows_seq
        self.plan = K.AttendPlan([rows_seq] * self.n, row0, 16, 512)
        self.d_row = torch.from_numpy(row0 + L).to(dev)
        self.d_pos = torch.full((self.n,), L, dtype=torch.int32, device=dev)
        nbytes = lib.kvl_mla_decode_step_workspace_bytes(C.byref(self.cfg), self.n)
        self.ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        self.units = self.LAYERS * self.rows * 1152  # attend bytes this rank reads per step
        self.total_bytes = self.LAYERS * seqs * L * 1152
        # per-launch DRAM traffic: the capture of one attend launch of the 16-sequence
        # slice of this step (profiles/mla_attend_bf16_config4.txt: 605.60 + 3.49 MB
        # for 524,304 rows), scaled by rows -- the kernel reads each row once
        self.ncu_traffic = {"mla_attend_bf16": (605.596928e6 + 3.485440e6) / 524304 * self.rows}

    def step_profiled(self):
        """The 27 decode steps launched one by one (per-kernel CUDA events)."""
        s = self.torch.cuda.current_stream().cuda_stream
        for layer in range(self.LAYERS):
            kv = self.kv[layer % self.nbuf]
            rc = self.lib.kvl_mla_decode_step_bf16(
                C.byref(self.cfg), C.byref(self.w[layer]), self.plan.h, self.out[layer].data_ptr(),
                self.x[layer].data_ptr(), kv.data_ptr(), self.rows, self.d_row.data_ptr(), self.d_pos.data_ptr(),
                self.n, self.ws.data_ptr(), s)
            if rc != 0:
                raise RuntimeError(self.K.last_error())

    def step(self):
        """One decode step of the stack as a CUDA graph of the 27 layer steps
        (captured once; every replay runs every kernel of every layer)."""
        replay_as_graph(self.torch, self, self.step_profiled, "decode_stack")

    def e2e_io(self):
        """Per step: the first layer's hidden states in, the last layer's out."""
        return [self.x[0]], [self.out[self.LAYERS - 1]]

    def value(self, ms):
        return self.total_bytes / (ms * 1e-3) / 1e9

    def config(self):
        return {"workload": "config 4: 27-layer batched decode step, 256 seqs x 32768 cached tokens",
                "seqs_per_rank": self.n, "layers": self.LAYERS, "layer_pools": self.nbuf,
                "pool_note": "all 27 layers resident" if self.nbuf == self.LAYERS else
                f"layer l reads pool l % {self.nbuf} (27 layers x 9.66 GB exceed one GPU)",
                "kv_bytes_per_step": self.total_bytes, "weights": "27 distinct layers, bf16 ~N(0,0.02)",
                "launch": ("the 27 layer steps captured once as a CUDA graph, replayed per step"
                           if getattr(self, "_graph", None) else "27 layer steps launched per step"),
                "parallelism": f"sequence-sharded x{self.dist.world}"}


class DecodeStackSlice(DecodeStack):
    """Config 4's decode step on 16 of its 256 sequences (the same 27 layers,
    shapes and kernels; a few GB on the device): the case whose attend launch
    is captured with ncu for config 4's DRAM traffic per row
    (profiles/mla_attend_bf16_config4.txt)."""
    name = "decode_stack_slice"
    metric = "MLA 27-layer decode KV GB/s (config 4 slice: 16 seqs x 32768)"

    def __init__(self, torch, K, lib, dist):
        # four layer pools of 0.6 GB (each far larger than L2), cycled by the 27 layers
        super().__init__(torch, K, lib, dist, seqs=16, max_pools=4)

    def config(self):
        cfg = super().config()
        cfg["workload"] = "config 4 slice: 27-layer decode step, 16 seqs x 32768 cached tokens"
        return cfg


class DecodeLongStack(DecodeStack):
    """Config 5's 27-layer variant: one decode step of the 27-layer text stack
    for one sequence at 131072 cached tokens (27 x 151 MB of bf16 KV, every
    layer resident), each layer a full kvl_mla_decode_step_bf16 whose attend
    splits the sequence over all SMs and merges the partials.  One GPU: the
    split-KV exchange across GPUs is the single-layer decode_long line."""
    name = "decode_long_stack"
    metric = "MLA 27-layer decode KV GB/s (config 5 variant: 1 seq x 131072)"

    def __init__(self, torch, K, lib, dist):
        super().__init__(torch, K, lib, dist, seqs=1, L=131072)

    def config(self):
        cfg = super().config()
        cfg["workload"] = "config 5, 27-layer variant: one decode step of the stack, 1 seq x 131072 cached tokens"
        cfg["parallelism"] = "one GPU"
        return cfg


class DecodeParity:
    """one sequence, 1024 cached rows, absorbed query
    [16,576] bf16 ~N(0,0.1), latent + rope bf16 ~N(0,1): the attend alone."""
    name = "decode_parity"
    metric = "MLA decode KV GB/s (config 1: 1 seq, L=1024)"
    unit = "GB/s"
    bound = "hbm"

    def __init__(self, torch, K, lib, dist, L=1024):
        self.torch, self.K, self.lib, self.dist = torch, K, lib, dist
        dev = torch.device("cuda", torch.cuda.current_device())
        g = torch.Generator(device=dev)
        g.manual_seed(1)
        self.L = L
        self.kv = dev_bf16(torch, (L, 576), 1.0, g, dev)
        self.q = dev_bf16(torch, (1, 16, 576), 0.1, g, dev).float()
        self.o = torch.empty((1, 16, 512), device=dev)
        self.plan = K.AttendPlan([L], [0], 16, 512)
        self.units = L * 1152
        self.total_bytes = dist.world * L * 1152

    def step(self):
        s = self.torch.cuda.current_stream().cuda_stream
        rc = self.plan.attend_bf16(self.o, None, self.q, self.kv, self.L, stream=s)
        if rc != 0:
            raise RuntimeError(self.K.last_error())

    def value(self, ms):
        return self.total_bytes / (ms * 1e-3) / 1e9

    def e2e_io(self):
        return [self.q], [self.o]

    def config(self):
        return {"workload": "config 1: single-sequence decode attend, L=1024", "rows": self.L,
                "parallelism": f"replicas x{self.dist.world}"}


def decode_e2e(torch, dist, wl, steps, warmup):
    """A decode sub-line end to end: every step copies the workload's inputs
    (e2e_io) from pinned host buffers to the device, runs the step (the same
    graph as the timed line) and reads its outputs back to pinned host
    buffers; host clock around the synchronised steps, max over ranks.  The KV
    state stays resident, as in a decoding runtime."""
    ins, outs = wl.e2e_io()
    h_in = [t.detach().cpu().pin_memory() for t in ins]
    h_out = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in outs]
    stream = torch.cuda.current_stream()

    def call():
        for d, h in zip(ins, h_in):
            d.copy_(h, non_blocking=True)
        wl.step()
        for d, h in zip(outs, h_out):
            h.copy_(d, non_blocking=True)
        stream.synchronize()
    for _ in range(warmup):
        call()
    dist.barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        call()
    dt = dist.max(torch, (time.perf_counter() - t0) * 1e3 / steps)
    nbytes = lambda ts: int(sum(t.numel() * t.element_size() for t in ts)) * dist.world  # noqa: E731
    return {"value": wl.value(dt), "unit": wl.unit, "ms_per_step": dt, "h2d_bytes_per_step": nbytes(ins),
            "d2h_bytes_per_step": nbytes(outs),
            "path": "per rank: inputs pinned host -> device, the step's launches, outputs device -> pinned host, "
                    "synchronised; bytes summed over ranks"}


def dropin_decode_line(K, lib, steps, warmup, cpu=True, lens=(1024, 8192)):
    """The call the reference runtime makes once per layer per token
    (src/generate.c:61): kvl_mla_decode_compressed_bf16 with host fp32 x and
    out in pageable memory (malloc'd, as the runtime's), against a state of L
    cached rows.  The call is synchronous, so each is timed on the host clock.
    Two weight modes: cached on the device by host pointer (what a full trunk
    cache allows, src/trunk_store.c:188-226) and uploaded on every call (the
    ~27.5 MB of one layer's projections, what the runtime's per-call weight
    reload implies otherwise, src/generate.c:40-76).  Beside each, the device
    time of the call's kernels (per-kernel CUDA events) and the reference's own
    call at the same L on this host's cores."""
    import kvl_b200.synth as SY
    cfg = K.make_config(2048, 16, 128, 64, 128, 512, 1e-5, 50000.0)
    w = K.random_weights(cfg, 1, 0.02)
    res = {"metric": "MLA drop-in decode latency (kvl_mla_decode_compressed_bf16, host fp32 x/out, pageable)",
           "unit": "ms/call", "h2d_bytes_per_call": {"x": 2048 * 4, "weights_when_uploaded": int(
               sum(a.nbytes for a in w.arrays))}, "d2h_bytes_per_call": {"out": 2048 * 4, "state_row_mirror": 576 * 4},
           "lengths": {}}
    prev = lib.kvl_mla_cuda_weight_cache(1)
    n = warmup + steps
    for L in lens:
        st = K.CompressedState(cfg, L + n + 1, lib=lib)
        x_pre = SY.bf16_bits_to_f32(SY.normal_bf16(11, SY.S_X, (L, 2048), 1.0))
        if st.prefill(x_pre, w) != 0:
            raise RuntimeError(K.last_error())
        xs = SY.bf16_bits_to_f32(SY.normal_bf16(12, SY.S_X, (n, 2048), 1.0))
        entry = {}
        for mode, cache in (("weights_cached", 1), ("weights_uploaded", 0)):
            lib.kvl_mla_cuda_weight_cache(cache)
            times = []
            for i in range(n):
                t0 = time.perf_counter()
                rc, _ = st.decode(xs[i], L + i, w)
                dt = time.perf_counter() - t0
                if rc != 0:
                    raise RuntimeError(K.last_error())
                if i >= warmup:
                    times.append(dt)
            if lib.kvl_mla_compressed_state_truncate(C.byref(st.s), L) != 0:
                raise RuntimeError(K.last_error())
            # device time of the same calls' kernels
            lib.kvl_mla_cuda_profile(1)
            for i in range(min(steps, 5)):
                st.decode(xs[i], L + i, w)
            prof = profile_read(lib)
            lib.kvl_mla_cuda_profile(0)
            if lib.kvl_mla_compressed_state_truncate(C.byref(st.s), L) != 0:
                raise RuntimeError(K.last_error())
            kern_ms = sum(v[0] for v in prof.values()) / max(1, min(steps, 5))
            entry[mode] = {"ms_per_call": 1e3 * float(np.median(times)), "ms_min": 1e3 * float(min(times)),
                           "kernel_ms_per_call": kern_ms,
                           "kernels_per_call": int(sum(v[1] for v in prof.values()) // max(1, min(steps, 5))),
                           "kv_gbs": L * 1152 / float(np.median(times)) / 1e9}
        st.free()
        if cpu:
            reps = 3 if L <= 2048 else 1
            dt = cpu_reference_decode(L, reps, 1) / reps
            entry["cpu_reference"] = {"ms_per_call": 1e3 * dt, "cores": host_threads(), "kind": "reference",
                                      "sample": f"reference kvl_mla_decode_compressed_bf16 (oracle/_ref, AVX2 + "
                                                f"OpenMP matvecs) at L={L}, mean of {reps} call(s)"}
            entry["speedup_vs_reference"] = {m: entry["cpu_reference"]["ms_per_call"] / entry[m]["ms_per_call"]
                                             for m in ("weights_cached", "weights_uploaded")}
        res["lengths"][str(L)] = entry
    lib.kvl_mla_cuda_weight_cache(prev)
    return res


def PrefillCP(torch, K, lib, dist):
    """Config 2 context-parallel at any N (N = 1: one rank holds both chunks)."""
    return Prefill(torch, K, lib, dist, mode="cp")


WORKLOADS = {"prefill": Prefill, "prefill_cp": PrefillCP, "decode_q8": DecodeQ8, "decode_q8_step": DecodeQ8Step,
             "decode_long": DecodeLong, "decode_long_stack": DecodeLongStack, "decode_stack": DecodeStack,
             "decode_parity": DecodeParity, "decode_stack_slice": DecodeStackSlice}


def measure(torch, K, lib, dist, wl, steps, warmup, flush, peaks):
    """Runs the timed loop, then a second profiled loop for the per-kernel
    durations of the dominant kernel (CUDA events on its launching stream)."""
    ms_total = timed_steps(torch, dist, wl.step, steps, warmup, flush)
    ms = ms_total / steps
    lib.kvl_mla_cuda_profile(1)
    for _ in range(steps):
        flush()
        getattr(wl, "step_profiled", wl.step)()
    torch.cuda.synchronize()
    prof = profile_read(lib)
    lib.kvl_mla_cuda_profile(0)
    wl.profiled_steps = steps
    launches = sum(c for _, c in prof.values()) // max(steps, 1)
    return ms, prof, launches


def roofline_for(wl, prof, peaks, peak_kind):
    """Dominant kernel = the library kernel with the largest device time."""
    if not prof:
        return None, None
    name, (tot_ms, cnt) = max(prof.items(), key=lambda kv: kv[1][0])
    per_launch_ms = tot_ms / max(cnt, 1)
    launches_per_step = max(1, round(cnt / max(1, getattr(wl, "profiled_steps", 1))))
    if wl.bound == "hbm":
        # one attend launch per step reads the rank's KV bytes once
        achieved = wl.units / launches_per_step / (per_launch_ms * 1e-3) / 1e9
        peak = peaks["hbm_gbs"]
        unit = "GB/s"
    else:
        algo_step = wl.kernel_flops().get(name, 0.0)
        achieved = algo_step / launches_per_step / (per_launch_ms * 1e-3) / 1e12
        peak = peaks["bf16_tflops"]
        unit = "TFLOP/s"
    traffic = getattr(wl, "ncu_traffic", {}).get(name) if getattr(wl, "dist", None) is None or \
        wl.dist.world == 1 else None
    return {"kernel": name, "bound": wl.bound, "achieved": achieved, "peak": peak, "unit": unit,
            "frac": achieved / peak, "peak_source": peak_kind, "ms_per_launch": per_launch_ms,
            "launches_measured": cnt, "traffic": traffic,
            "traffic_unit": "bytes per launch (ncu dram read+write)" if traffic is not None else None}, name


# ----------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="prefill")
    ap.add_argument("--no-extras", action="store_true", help="skip the decode sub-measurements")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end (host buffer) leg")
    args = ap.parse_args()
    dist = Dist()

    if args.impl == "reference":
        return run_reference(args, dist)

    import torch
    dist.init(torch)
    K, lib = load_lib()
    peaks, peak_kind = load_peaks()
    dev = torch.device("cuda", torch.cuda.current_device())
    flush_buf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def flush():
        flush_buf.fill_(1)

    wl = WORKLOADS[args.workload](torch, K, lib, dist)
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    ms, prof, launches = measure(torch, K, lib, dist, wl, args.steps, args.warmup, flush, peaks)
    clk = clocks.stop()
    roof, dom = roofline_for(wl, prof, peaks, peak_kind)
    line = {
        "metric": wl.metric, "value": wl.value(ms), "unit": wl.unit, "n_gpus": dist.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": getattr(wl, "scaling", "strong"), "vs_baseline": None, "dtype": getattr(wl, "dtype", "bf16"),
        "data": "synthetic (seeded)",
        "config": wl.config(), "launch": wl.launch() if hasattr(wl, "launch") else None,
        "roofline": roof, "gpu_launches": int(launches) * args.steps,
        "kernels": {k: {"ms_total": v[0], "launches": v[1]} for k, v in prof.items()}, "clocks": clk,
    }
    if hasattr(wl, "e2e") and not args.no_e2e:
        line["e2e"] = wl.e2e(max(2, args.steps // 2), 1)
    if not args.no_extras and args.workload == "prefill":
        extras = {}
        names = ("decode_parity", "decode_q8", "decode_q8_step", "decode_long", "decode_stack")
        if dist.world > 1:  # beside the context-parallel headline: one independent prompt per GPU
            names = ("prefill_independent",) + names
        else:  # config 5's 27-layer variant (one GPU)
            names = names + ("decode_long_stack",)
        for name in names:
            w2, err = None, None
            try:
                if name == "prefill_independent":
                    w2 = Prefill(torch, K, lib, dist, mode="independent")
                else:
                    w2 = WORKLOADS[name](torch, K, lib, dist)
            except Exception as e:  # noqa: BLE001 - report, keep the headline
                err = str(e)
            # every rank takes the same collective steps: skip on all ranks if any failed to set up
            if dist.sum(torch, 0.0 if err is None else 1.0) > 0:
                extras[name] = {"error": err or "set-up failed on another rank"}
                del w2
                torch.cuda.empty_cache()
                continue
            ms2, prof2, l2 = measure(torch, K, lib, dist, w2, args.steps, args.warmup, flush, peaks)
            r2, _ = roofline_for(w2, prof2, peaks, peak_kind)
            extras[name] = {"metric": w2.metric, "value": w2.value(ms2), "unit": w2.unit, "ms_per_step": ms2,
                            "dtype": getattr(w2, "dtype", "bf16"),
                            "frac_of_peak": w2.value(ms2) / ((peaks["hbm_gbs"] if w2.unit == "GB/s" else
                                                              peaks["bf16_tflops"]) * dist.world),
                            "roofline": r2,
                            "config": w2.config(), "gpu_launches_per_step": int(l2),
                            "kernels": {k: {"ms_total": v[0], "launches": v[1]} for k, v in prof2.items()}}
            if hasattr(w2, "e2e_io") and not args.no_e2e:
                extras[name]["e2e"] = decode_e2e(torch, dist, w2, max(2, args.steps // 2), 1)
            if dist.rank == 0 and dist.world == 1 and not args.no_cpu:
                cb = decode_cpu_baseline(name, w2)
                if cb is not None:
                    extras[name]["cpu_baseline"] = cb
            del w2
            torch.cuda.empty_cache()
        if dist.rank == 0 and dist.world == 1:
            try:
                extras["decode_dropin"] = dropin_decode_line(K, lib, max(5, args.steps), 3, cpu=not args.no_cpu)
            except Exception as e:  # noqa: BLE001
                extras["decode_dropin"] = {"error": str(e)}
        line["decode"] = extras
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu and hasattr(wl, "cpu_baseline"):
        try:
            line["cpu_baseline"] = wl.cpu_baseline()
        except Exception as e:  # noqa: BLE001
            line["cpu_baseline"] = {"error": str(e)}
    if dist.rank == 0:
        print(json.dumps(line), flush=True)
    dist.close()
    return 0


def run_reference(args, dist):
    """The reference's own CPU implementation of the path on this host's cores
    (oracle/_ref: the reference sources compiled with AVX2 + OpenMP).  Under
    torchrun only rank 0 runs; the others exit without work."""
    if dist.rank != 0:
        return 0
    # every host thread this process may use (torchrun exports OMP_NUM_THREADS=1
    # to each rank; here rank 0 runs alone), set before the reference library
    # and its OpenMP runtime are loaded
    try:
        cores = len(os.sched_getaffinity(0))
    except AttributeError:
        cores = os.cpu_count() or 1
    os.environ["OMP_NUM_THREADS"] = str(cores)
    from oracle.oracle import reference_available
    if not reference_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref was not built (reference sources absent)"}))
        return 0
    if args.workload != "prefill":
        print(json.dumps({"impl": "reference", "unavailable": f"reference arm implemented for prefill only"}))
        return 0
    S = 4096
    prefill_inputs(S)
    for _ in range(max(0, min(args.warmup, 1))):
        cpu_reference_prefill(S)
    times, fl = [], 0
    for _ in range(args.steps):
        dt, fl = cpu_reference_prefill(S)
        times.append(dt)
    ms = 1e3 * sum(times) / len(times)
    value = fl / (ms * 1e-3) / 1e12
    sample = (f"reference kvl_mla_prefill_bf16 (AVX2+OpenMP, {cores} threads) on one {S}-token sequence at config-2 "
              f"shapes per step ({fl / 1e9:.2f} GFLOP): the full config-2 workload")
    print(json.dumps({
        "impl": "reference", "metric": Prefill.metric, "value": value, "unit": Prefill.unit, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 (bf16 weights)", "data": "synthetic (seeded)",
        "config": prefill_config(S, 50000.0, args.gpus),
        "launch": f"reference kvl_mla_prefill_bf16 on the host ({cores} threads), one call per step",
        "cpu_baseline": {"value": value, "unit": Prefill.unit, "cores": cores, "kind": "reference", "sample": sample},
        "e2e": {"value": value, "unit": Prefill.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
