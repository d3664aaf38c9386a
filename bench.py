#!/usr/bin/env python
"""Paged K/V gather + append throughput on the Qwen-Image-2.1 1K-edit workload (B200).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step is one edit turn of the 1K config: the 4608-token cached prefix (512 text + 4096 conditioning-image
tokens; 60 layers, 24 heads x 128, bf16, page 64, 24 GiB pool) is gathered for each of the 8 denoising steps,
then the turn's 4096 new image tokens are appended (alloc + write + insert). Sessions are partitioned over
GPUs (one process per GPU, no collective on the data path; `scaling: weak`).

* ``value``  device-resident throughput: the turn's kernel launches (8 gathers + 1 append) replayed on
  slot tables prepared before the timed region; CUDA events, max over ranks.
* ``e2e``    the same turns through the public pool API (host prefix index, slot tables copied to the
  device, kernels, and a device-to-host read of the turn's result probe).
* ``roofline`` the gather kernel's algorithmic bytes / its CUDA-event launch time vs the measured HBM copy
  bandwidth; DRAM traffic from the committed ncu summary.
* ``cpu_baseline`` / ``--impl reference``: the reference's own torch ops (index_select / index_copy_) with the
  restated prefix index on the host CPU, on a bounded sample (8 of the 60 layers).
Inputs are far larger than L2 (6.8 GB per gather), so no L2 flush is needed between iterations.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "paged K/V gather+append HBM GB/s (% peak); DiT step ms at 1K/2K edit"
L, H, D, PAGE = 60, 24, 128, 64
TEXT, IMAGE, APPEND, STEPS_PER_TURN = 512, 4096, 4096, 8
PREFIX = TEXT + IMAGE
POOL_GIB = 24
ROW = H * D * 2  # bytes of one token's K (or V) in one layer
GATHER_BYTES = 2 * L * 2 * PREFIX * ROW + (PREFIX // PAGE) * 4
APPEND_BYTES = 2 * L * 2 * APPEND * ROW + (APPEND // PAGE) * 4
TURN_BYTES = STEPS_PER_TURN * GATHER_BYTES + APPEND_BYTES
CPU_SAMPLE_LAYERS = 8
CONFIG = {
    "workload": "qwen_image_2.1_1k_edit_paged_prefix_kv",
    "layers": L, "heads": H, "head_dim": D, "dtype": "bf16", "page_tokens": PAGE, "pool_gib": POOL_GIB,
    "prefix_tokens": PREFIX, "append_tokens": APPEND, "gathers_per_turn": STEPS_PER_TURN,
    "block_tables": "seeded random page permutation (shuffled free list)",
    "l2": "no flush: each gather moves 6.8 GB, >> 126 MB L2",
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the 2K and NVFP4 side measurements")
    ap.add_argument("--workload", choices=["edit_1k", "serving", "headshard"], default="edit_1k",
                    help="edit_1k: the 1K-edit turn (default, the headline); serving: 64 mixed 1K/2K sessions")
    ap.add_argument("--profile", choices=["gather", "append", "norm", "silu", "short_rows", "attention", "gather_heads",
                                                   "mask_blend", "norm_amax", "silu_amax"], default=None,
                    help="small case for ncu: 3 warm-up + 3 launches of one kernel (a few GB on the device)")
    return ap.parse_args()


# ---- clocks ------------------------------------------------------------------------------------
class ClockSampler(threading.Thread):
    """Samples SM clock and clock-event reasons through NVML (read-only) while the timed region runs."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting", 0x1: "gpu_idle"}

    def __init__(self, device: int):
        super().__init__(daemon=True)
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._halt = threading.Event()
        self.ok = False
        try:
            import pynvml

            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            try:
                self.h = pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + uuid) if not uuid.startswith("GPU-") else uuid)
            except Exception:
                self.h = pynvml.nvmlDeviceGetHandleByIndex(device)
            self.nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as exc:  # no NVML: report nothing rather than guess
            self.err = str(exc)

    def run(self):
        while self.ok and not self._halt.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                getter = getattr(self.nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                    self.nv.nvmlDeviceGetCurrentClocksThrottleReasons
                bits = getter(self.h)
                for bit, name in self.REASONS.items():
                    if bits & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.01)  # ~10 samples over a 0.1 s timed region

    def stop(self) -> dict:
        self._halt.set()
        if self.is_alive():
            self.join(timeout=2)
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        return {"sm_mhz": float(statistics.median(self.samples)), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def measured_peak() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, copy burst)"
    except Exception:
        return 6650.0, "fallback (6.65 TB/s pool figure)"


def committed_traffic(kernel: str) -> dict | None:
    """DRAM bytes per launch of `kernel` from the committed ncu summary (profiles/traffic.txt): read and write
    separately (the write count is a lower bound: lines still dirty in L2 when the kernel ends are not counted)."""
    path = ROOT / "profiles" / "traffic.txt"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 3 and parts[0] == kernel:
            try:
                return {"read": float(parts[1]), "write": float(parts[2])}
            except ValueError:
                return None
    return None


# ---- distributed plumbing ----------------------------------------------------------------------
def dist_setup(args):
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if world > 1:
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=120),
                                              device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ---- the workload --------------------------------------------------------------------------------
class Session:
    """One edit session on one GPU: text header + a new conditioning image per turn."""

    def __init__(self, pool, seed: int, device):
        from qwenedit_b200 import keys

        self.pool, self.device = pool, device
        self.rng = np.random.default_rng(seed)
        root = keys.root_key("dit", "Qwen/Qwen-Image-2.1", "bench", seed)
        prev = int.from_bytes(root[:8], "little") & ((1 << 63) - 1)
        self.text = np.empty(TEXT, np.int64)
        for i, tok in enumerate(self.rng.integers(0, 150_000, size=TEXT)):
            prev = keys.text_id(prev, int(tok))
            self.text[i] = prev
        self.turn = 0
        self.new_kv = torch.empty(L, 2, APPEND, H, D, dtype=torch.bfloat16, device=device)
        self.new_kv.normal_()
        self.out = torch.empty(L, 2, PREFIX, H, D, dtype=torch.bfloat16, device=device)
        # turn 0's prefix was computed by the DiT on a miss (hooks.py:126-139): store it whole
        first = self.vids(0)
        slots = pool.alloc(PREFIX)
        pool.write(slots, torch.randn(L, 2, PREFIX, H, D, dtype=torch.bfloat16, device=device))
        pool.insert(first, slots, owned_from=0)

    def image_ids(self, turn: int) -> np.ndarray:
        from qwenedit_b200 import keys

        content = b"img" + turn.to_bytes(8, "little") + np.asarray([64, 64], np.int64).tobytes()
        return keys.block_ids(int(self.text[-1]), content, IMAGE)

    def vids(self, turn: int) -> np.ndarray:
        return np.concatenate([self.text, self.image_ids(turn)])

    def api_turn(self, gather_events=None):
        """One turn through the public pool API; returns the prefix Match (released) and the appended slots."""
        pool = self.pool
        m = pool.match(self.vids(self.turn))
        if m.length != PREFIX:
            raise RuntimeError(f"turn {self.turn}: expected a full prefix hit, got {m.length}")
        for s in range(STEPS_PER_TURN):
            if gather_events is not None:
                gather_events[s][0].record()
            pool.gather_into(m.indices, self.out)
            if gather_events is not None:
                gather_events[s][1].record()
        slots = pool.alloc(APPEND)
        if slots is None:
            raise RuntimeError("pool exhausted")
        pool.write(slots, self.new_kv)
        nxt = self.vids(self.turn + 1)
        idx_host = np.concatenate([m.indices._qe_host[:TEXT], slots._qe_host])
        idx = torch.from_numpy(idx_host)
        idx._qe_host = idx_host
        pool.insert(nxt, idx, owned_from=TEXT)
        m.release()
        self.turn += 1
        return m, slots


def run_ours(args, rank, world, local):
    from qwenedit_b200.paged import PagedKVPool

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    pool = PagedKVPool("dit", L, H, D, POOL_GIB << 30, torch.bfloat16, device, page_size=PAGE)
    pool.index.shuffle_free(1000 + rank)
    pool.kv.normal_()
    sess = Session(pool, seed=rank, device=device)
    stream = torch.cuda.current_stream(device)

    # ---- value: device-resident replay of K turns -------------------------------------------------
    # host bookkeeping (match / alloc / insert) for warm-up + timed turns is done up front; the timed region
    # launches exactly the turns' kernels on their slot tables (already on the device)
    plans = []
    for _ in range(args.warmup + args.steps):
        m = pool.match(sess.vids(sess.turn))
        assert m.length == PREFIX
        pool._block_table(m.indices, m.indices._qe_host)
        slots = pool.alloc(APPEND)
        pool._block_table(slots, slots._qe_host)
        idx_host = np.concatenate([m.indices._qe_host[:TEXT], slots._qe_host])
        idx = torch.from_numpy(idx_host)
        idx._qe_host = idx_host
        pool.insert(sess.vids(sess.turn + 1), idx, owned_from=TEXT)
        m.release()
        sess.turn += 1
        plans.append((m.indices, slots))
    torch.cuda.synchronize()

    def replay(plan, ev=None):
        prefix_slots, append_slots = plan
        for s in range(STEPS_PER_TURN):
            if ev is not None:
                ev[s][0].record(stream)
            pool.gather_into(prefix_slots, sess.out)
            if ev is not None:
                ev[s][1].record(stream)
        pool.write(append_slots, sess.new_kv)

    for plan in plans[: args.warmup]:
        replay(plan)
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    barrier(world)
    torch.cuda.synchronize()
    launch_events = [[[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(STEPS_PER_TURN)]
                     for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for k, plan in enumerate(plans[args.warmup:]):
        replay(plan, launch_events[k])
    t1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clock_info = clocks.stop()
    elapsed_ms = max_over_ranks(t0.elapsed_time(t1), world, device)
    gather_ms = [ev[0].elapsed_time(ev[1]) for turn in launch_events for ev in turn]
    avg_gather_ms = max_over_ranks(statistics.mean(gather_ms), world, device)
    if pool.device_errors():
        raise RuntimeError("a kernel reported an out-of-range slot")

    # ---- e2e: the same turns through the public API; every turn's result probe (the pool's device error flag
    # and 8 bytes of the last gathered row) is copied to pinned host memory and read back, one turn behind so the
    # host bookkeeping of turn t+1 overlaps the device work of turn t, as a serving loop would run it
    probes = [torch.empty(2, dtype=torch.int64, pin_memory=True) for _ in range(2)]

    def issue_probe(k):
        probe_dev = torch.stack([pool._err.to(torch.int64)[0], sess.out[-1, 1, -1, -1, -4:].view(torch.int64)[0]])
        probes[k % 2].copy_(probe_dev, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(stream)
        return ev

    def read_probe(k, ev):
        ev.synchronize()
        if int(probes[k % 2][0]) != 0:
            raise RuntimeError("device error flag set")

    for k in range(args.warmup):
        sess.api_turn()
        read_probe(k, issue_probe(k))
    torch.cuda.synchronize()
    h2d0 = pool.h2d_bytes
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    wall0 = time.perf_counter()
    pending = None
    for k in range(args.steps):
        sess.api_turn()
        ev = issue_probe(k)
        if pending is not None:
            read_probe(*pending)
        pending = (k, ev)
    read_probe(*pending)
    e1.record(stream)
    torch.cuda.synchronize()
    wall_ms = (time.perf_counter() - wall0) * 1e3
    barrier(world)
    e2e_ms = max_over_ranks(max(e0.elapsed_time(e1), wall_ms), world, device)
    h2d_per_step = (pool.h2d_bytes - h2d0) / args.steps
    d2h_per_step = probes[0].numel() * probes[0].element_size()

    result = {}
    if not args.no_extras and world == 1:  # side measurements are per-GPU; the scaling runs skip them
        result = extras(pool, sess, device)
    return dict(elapsed_ms=elapsed_ms, avg_gather_ms=avg_gather_ms, clocks=clock_info, e2e_ms=e2e_ms,
                h2d=h2d_per_step, d2h=d2h_per_step, extras=result)


def extras(pool, sess, device):
    """Side measurements (outside the headline): DiT step gather at 2K, NVFP4 kernels."""
    from qwenedit_b200.paged import set_copy_mode

    out = {}
    peak, _ = measured_peak()
    # the paged-copy kernels (warp copy with 256-bit or 16-byte vectors, TMA bulk) on the 1K turn's gather and append
    m = pool.match(sess.vids(sess.turn))
    slots = pool.alloc(APPEND)
    variants = {}
    for mode in ("warp", "warp16", "bulk"):
        set_copy_mode(mode)
        g_ms = _time_kernel(lambda: pool.gather_into(m.indices, sess.out), None, iters=5)
        a_ms = _time_kernel(lambda: pool.write(slots, sess.new_kv), None, iters=5)
        variants[mode] = {"gather_ms": round(g_ms, 4), "gather_GB/s": round(GATHER_BYTES / g_ms / 1e6, 1),
                          "gather_frac": round(GATHER_BYTES / g_ms / 1e6 / peak, 4),
                          "append_ms": round(a_ms, 4), "append_GB/s": round(APPEND_BYTES / a_ms / 1e6, 1),
                          "append_frac": round(APPEND_BYTES / a_ms / 1e6 / peak, 4)}
    set_copy_mode("auto")
    m.release()
    out["paged_copy_kernels_1k"] = variants
    if pool.device_errors():
        raise RuntimeError("a paged copy kernel reported an error")
    # 2K edit: 16384 cond-image + 512 text prefix tokens, per-step gather through a random block table
    pool.clear()
    pool.index.shuffle_free(7)
    T2 = 16384 + 512
    vids = np.arange(1, T2 + 1, dtype=np.int64) + (1 << 40)
    slots = pool.alloc(T2)
    pool.insert(vids, slots, owned_from=0)
    m = pool.match(vids)
    big = torch.empty(L, 2, T2, H, D, dtype=torch.bfloat16, device=device)
    for _ in range(2):
        pool.gather_into(m.indices, big)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(5)]
    for a, b in ev:
        a.record()
        pool.gather_into(m.indices, big)
        b.record()
    torch.cuda.synchronize()
    ms2k = statistics.mean(a.elapsed_time(b) for a, b in ev)
    bytes2k = 2 * L * 2 * T2 * ROW
    out["dit_step_gather_2k"] = {"prefix_tokens": T2, "ms": round(ms2k, 4), "GB/s": round(bytes2k / ms2k / 1e6, 1),
                                 "frac_of_measured_hbm": round(bytes2k / ms2k / 1e6 / peak, 4)}
    m.release()
    del big
    torch.cuda.empty_cache()
    out["paged_attention_1k"] = attention_extras(pool, device)
    out.update(nvfp4_extras(device, peak))
    out["nvfp4_cpu_baseline"] = nvfp4_cpu()
    out["mask_blend_1k"] = latent_extras(device)
    out["encoder_prompt_1k"] = encoder_extras(device, peak)
    out["prefix_index_host_latency_1k"] = index_latency()
    return out


def index_latency(turns: int = 40, page: int = PAGE) -> dict:
    """Host latency of the prefix index per 1K-edit turn (reported as latency, not bandwidth):
    match of the 4,608-token prefix, alloc of the 4,096 new tokens (with LRU eviction once the 24 GiB pool is
    full), insert of the next prefix, release. The native index (libqeb200) against the oracle's Python
    restatement of the reference's tree (SGLang RadixCache + allocator), both index-only (no device data)."""
    from oracle.pool_ref import RefPagedKVPool
    from qwenedit_b200.paged import PagedKVPool

    budget = POOL_GIB << 30
    ours = PagedKVPool("idx", L, H, D, budget, torch.bfloat16, "meta", page_size=page)
    ref = RefPagedKVPool("idx", L, H, D, budget, torch.bfloat16, page_size=page, allocate=False)
    rng = np.random.default_rng(4)
    text = rng.integers(1, 1 << 62, size=TEXT)
    images = [rng.integers(1, 1 << 62, size=IMAGE) for _ in range(turns + 2)]
    out = {}
    for name, pool in (("native", ours), ("python_reference_tree", ref)):
        first = np.concatenate([text, images[0]])
        s0 = pool.alloc(PREFIX)
        pool.insert(first, s0, owned_from=0)
        t = {"match": [], "alloc": [], "insert": [], "release": []}
        for turn in range(turns):
            a = time.perf_counter()
            m = pool.match(np.concatenate([text, images[turn]]))
            b = time.perf_counter()
            slots = pool.alloc(APPEND)
            c = time.perf_counter()
            host = np.concatenate([np.asarray(m.indices[:TEXT].numpy() if not hasattr(m.indices, "_qe_host")
                                              else m.indices._qe_host[:TEXT]), np.asarray(
                slots._qe_host if hasattr(slots, "_qe_host") else slots.numpy())])
            idx = torch.from_numpy(host.copy())
            idx._qe_host = idx.numpy()
            d = time.perf_counter()
            pool.insert(np.concatenate([text, images[turn + 1]]), idx, owned_from=TEXT)
            e = time.perf_counter()
            m.release()
            f = time.perf_counter()
            for k, v in (("match", b - a), ("alloc", c - b), ("insert", e - d), ("release", f - e)):
                t[k].append(v * 1e6)
        out[name] = {k: round(statistics.median(v), 1) for k, v in t.items()}
        out[name]["evicted_tokens"] = int(pool.usage()["evicted_tokens"] if hasattr(pool, "usage") else 0)
    out["unit"] = "us per call (median over turns)"
    return out


def encoder_extras(device, peak):
    """Text-encoder pool (Qwen2.5-VL: 28 layers, 4 KV heads x 128, hidden 3584; 4 GiB, token-granular slots):
    a full hit of a 1,024-token prompt returns the hidden rows (encoder.py:114), a partial hit gathers the
    prefix K/V (encoder.py:173). Single launches between CUDA events after an L2 flush, scattered slots."""
    from qwenedit_b200.paged import PagedKVPool

    layers, kvh, hd, hidden, n = 28, 4, 128, 3584, 1024
    pool = PagedKVPool("encoder", layers, kvh, hd, 4 << 30, torch.bfloat16, device, extra_dim=hidden)
    pool.index.shuffle_free(77)
    slots = pool.alloc(n)
    pool.write(slots, torch.randn(layers, 2, n, kvh, hd, device=device).bfloat16())
    pool.write_extra(slots, torch.randn(n, hidden, device=device).bfloat16())
    out_kv = torch.empty(layers, 2, n, kvh, hd, dtype=torch.bfloat16, device=device)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    kv_ms = _time_kernel(lambda: pool.gather_into(slots, out_kv), flush)
    hid_ms = _time_kernel(lambda: pool.gather_extra(slots), flush)
    kv_bytes = 2 * layers * 2 * n * kvh * hd * 2
    hid_bytes = 2 * n * hidden * 2
    # partial hit (encoder.py:173-182): the prefix K/V head-major with room for a 256-token tail, in one launch,
    # against the reference's gather followed by a transpose + cat per layer and K/V (torch ops on our gather)
    tail = 256
    k_tail = torch.randn(1, kvh, tail, hd, device=device).bfloat16()

    def ours():
        buf = pool.gather_heads(slots, n + tail)
        for layer in range(layers):
            buf[layer, 0, :, n:] = k_tail[0]
            buf[layer, 1, :, n:] = k_tail[0]

    def reference_ops():
        cached = pool.gather(slots)
        for layer in range(layers):
            torch.cat([cached[layer, 0].transpose(0, 1)[None], k_tail], dim=2)
            torch.cat([cached[layer, 1].transpose(0, 1)[None], k_tail], dim=2)

    tail_ms = _time_graph([ours])
    tail_ref_ms = _time_graph([reference_ops])
    # the partial hit's attention (encoder.py:173-190): 28 query heads over [prefix; tail] with the reference's
    # tril(diagonal=m) mask, every layer: the paged kernel over the head-major gather (token-granular pool) against
    # the reference's gather + per-layer transpose / cat + masked GQA SDPA
    import torch.nn.functional as F

    from qwenedit_b200.attention import encoder_tail_attention

    hq, scale = 28, hd ** -0.5
    q_t = torch.randn(tail, hq, hd, device=device).bfloat16()
    kv_t = torch.randn(2, tail, kvh, hd, device=device).bfloat16()
    heads_out = torch.empty(tail, hq, hd, dtype=torch.bfloat16, device=device)
    mask = torch.ones(tail, n + tail, dtype=torch.bool, device=device).tril(diagonal=n)

    def ours_attention():
        buf = pool.gather_heads(slots, n + tail)
        for layer in range(layers):
            heads_out.copy_(encoder_tail_attention(q_t, kv_t[0], kv_t[1], pool, slots, layer, scale, heads_buf=buf))

    def reference_attention():
        cached = pool.gather(slots)
        for layer in range(layers):
            k = torch.cat([cached[layer, 0].transpose(0, 1)[None], kv_t[0].transpose(0, 1)[None]], dim=2)
            v = torch.cat([cached[layer, 1].transpose(0, 1)[None], kv_t[1].transpose(0, 1)[None]], dim=2)
            F.scaled_dot_product_attention(q_t.transpose(0, 1)[None], k, v, attn_mask=mask, scale=scale,
                                           enable_gqa=True)

    att_ms = _time_graph([ours_attention])
    try:
        att_ref_ms = _time_graph([reference_attention])
    except Exception:  # noqa: BLE001  (a torch build whose masked GQA SDPA does not capture)
        att_ref_ms = None
    # steady state: 8 prompts' gathers back to back from one CUDA graph (cycled to GRAPH_LAUNCHES launches), each
    # prompt's own scattered slots and output (0.94 GB of K/V in total, > L2), so every launch reads HBM and no
    # launch latency is in the time; also the partial hit's head-major gather (room for the 256-token tail)
    prompts = [pool.alloc(n) for _ in range(8)]
    outs = [torch.empty_like(out_kv) for _ in prompts]
    kv_ss_ms = _time_graph([lambda s_=s_, o=o: pool.gather_into(s_, o) for s_, o in zip(prompts, outs)],
                           min_launches=GRAPH_LAUNCHES)
    hid_ss_ms = _time_graph([lambda s_=s_: pool.gather_extra(s_) for s_ in prompts], min_launches=GRAPH_LAUNCHES)
    heads_ss_ms = _time_graph([lambda s_=s_: pool.gather_heads(s_, n + tail) for s_ in prompts],
                              min_launches=GRAPH_LAUNCHES)
    if pool.device_errors():
        raise RuntimeError("encoder gather reported an error")
    return {"kv_gather_ms": round(kv_ms, 4), "kv_GB/s": round(kv_bytes / kv_ms / 1e6, 1),
            "hidden_gather_ms": round(hid_ms, 4), "hidden_GB/s": round(hid_bytes / hid_ms / 1e6, 1),
            "bytes": {"kv": kv_bytes, "hidden": hid_bytes}, "note": "single launches: launch latency included",
            "steady_state": {"kv_gather_ms": round(kv_ss_ms, 4), "kv_GB/s": round(kv_bytes / kv_ss_ms / 1e6, 1),
                             "kv_frac_of_measured_hbm": round(kv_bytes / kv_ss_ms / 1e6 / peak, 4),
                             "hidden_gather_ms": round(hid_ss_ms, 4),
                             "hidden_GB/s": round(hid_bytes / hid_ss_ms / 1e6, 1),
                             "hidden_frac_of_measured_hbm": round(hid_bytes / hid_ss_ms / 1e6 / peak, 4),
                             "head_major_kv_gather_ms": round(heads_ss_ms, 4),
                             "head_major_kv_GB/s": round(kv_bytes / heads_ss_ms / 1e6, 1),
                             "head_major_kv_frac_of_measured_hbm": round(kv_bytes / heads_ss_ms / 1e6 / peak, 4),
                             "timing": f"8 prompts back to back from one CUDA graph ({GRAPH_LAUNCHES} launches), "
                                       "per-launch mean"},
            "partial_hit_prefix_ms": {"gather_heads_plus_tail_writes": round(tail_ms, 4),
                                      "gather_then_per_layer_transpose_cat": round(tail_ref_ms, 4),
                                      "prefix_tokens": n, "tail_tokens": tail, "timing": "CUDA graph, device time"},
            "partial_hit_attention_ms": {"gather_heads_then_paged_attention": round(att_ms, 4),
                                         "gather_cat_masked_gqa_sdpa": None if att_ref_ms is None else
                                         round(att_ref_ms, 4),
                                         "layers": layers, "query_heads": hq, "kv_heads": kvh, "prefix_tokens": n,
                                         "tail_tokens": tail, "timing": "CUDA graph, device time, all layers"}}


def latent_extras(device):
    """Per-step mask blend on 1K latents [1, 4096, 64] bf16, one launch (the reference's eager blend is about ten
    launches): device time per call from a CUDA graph of 100 calls (no host time in it), and the host time of an
    eager call."""
    from qwenedit_b200.latents import mask_blend

    lat = torch.randn(1, 4096, 64, device=device).bfloat16()
    x0, eps = torch.randn_like(lat), torch.randn_like(lat)
    m = torch.rand(1, 4096, 1, device=device)
    sigma = torch.tensor(0.5, device=device)
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        for _ in range(5):
            mask_blend(lat, x0, eps, m, sigma)
    torch.cuda.current_stream(device).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(100):
            mask_blend(lat, x0, eps, m, sigma)
    graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    graph.replay()
    b.record()
    torch.cuda.synchronize()
    device_us = a.elapsed_time(b) / 100 * 1e3
    t0 = time.perf_counter()
    for _ in range(200):
        mask_blend(lat, x0, eps, m, sigma)
    host_us = (time.perf_counter() - t0) / 200 * 1e6
    torch.cuda.synchronize()
    del graph
    nbytes = 4 * lat.numel() * 2 + m.numel() * 4
    return {"device_us_per_call": round(device_us, 2), "host_us_per_call": round(host_us, 1),
            "launches_per_call": 1, "bytes_per_call": nbytes,
            "GB/s": round(nbytes / device_us / 1e3, 1)}


def attention_extras(pool, device):
    """One DiT step's joint attention at the 1K edit (60 layers; 4096 latent queries over the 4608-token pooled
    prefix, page 64 through a shuffled block table, plus their own 4096 keys; 24 heads x 128): the paged kernel
    (qe_paged_attention, one launch per layer, prefix read from the pool pages) against the path it replaces, one
    gather of the prefix for all layers followed per layer by a concatenation with the own K/V and torch's SDPA
    (cuDNN backend, the fastest library attention on this GPU). FLOPs per layer 4 n_q (n_prefix + n_own) D H."""
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    from qwenedit_b200.attention import PagedPrefix, paged_attention

    pool.clear()
    pool.index.shuffle_free(11)
    vids = np.arange(1, PREFIX + 1, dtype=np.int64) + (1 << 41)
    slots = pool.alloc(PREFIX)
    pool.insert(vids, slots, owned_from=0)
    m = pool.match(vids)
    prefix = PagedPrefix(pool, m.indices)
    n = IMAGE
    g = torch.Generator(device=device).manual_seed(0)
    q, k_own, v_own = (torch.randn(n, H, D, generator=g, device=device).bfloat16() for _ in range(3))
    out = torch.empty(n, H, D, dtype=torch.bfloat16, device=device)
    flops_layer = 4.0 * n * (PREFIX + n) * D * H

    def ours():
        for layer in range(L):
            paged_attention(q, prefix, layer, k_own, v_own, out=out)

    gathered = torch.empty(L, 2, PREFIX, H, D, dtype=torch.bfloat16, device=device)
    qh = q.transpose(0, 1)[None]

    def gather_then_sdpa():
        pool.gather_into(m.indices, gathered)
        for layer in range(L):
            k = torch.cat([gathered[layer, 0], k_own]).transpose(0, 1)[None]
            v = torch.cat([gathered[layer, 1], v_own]).transpose(0, 1)[None]
            with sdpa_kernel(SDPBackend.CUDNN_ATTENTION):
                F.scaled_dot_product_attention(qh, k, v)

    def timed(fn, reps=3):
        fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b))
        return statistics.median(ts)

    ms = timed(ours)
    try:
        ms_ref = timed(gather_then_sdpa)
    except Exception:  # noqa: BLE001  (no cuDNN attention in this torch build)
        ms_ref = None
    # the own K/V also stored into freshly allocated pool pages (a prefill tail, or the encoder's _store): in the
    # attention launch itself (qe_paged_attention_append) against the attention then one write_layers launch
    appended = None
    tail_slots = pool.alloc(n)
    if tail_slots is not None:
        app = PagedPrefix(pool, tail_slots)
        keys, values = [k_own] * L, [v_own] * L

        def ours_append():
            for layer in range(L):
                paged_attention(q, prefix, layer, k_own, v_own, out=out, append=app)

        def ours_then_write():
            ours()
            pool.write_layers(tail_slots, keys, values)

        ms_app, ms_sep = timed(ours_append), timed(ours_then_write)
        appended = {"tokens": n, "bytes_per_step": L * 2 * n * H * D * 2, "ms_per_step": round(ms_app, 3),
                    "attention_then_write_layers_ms_per_step": round(ms_sep, 3),
                    "append_cost_ms_per_step": round(ms_app - ms, 3)}
    if pool.device_errors():
        raise RuntimeError("the paged attention kernel reported an error")
    peaks = {}
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        peaks = json.loads(path.read_text())
    tf = flops_layer * L / ms / 1e9
    res = {"layers": L, "queries": n, "prefix_tokens": PREFIX, "own_tokens": n, "heads": H,
           "ms_per_step": round(ms, 3), "ms_per_layer": round(ms / L, 4), "TFLOP/s": round(tf, 1),
           "gather_then_cudnn_sdpa_ms_per_step": None if ms_ref is None else round(ms_ref, 3),
           "speedup_vs_gather_then_cudnn_sdpa": None if ms_ref is None else round(ms_ref / ms, 3),
           "timing": "CUDA events around one step's 60 launches (inputs resident, 2.3 GB of prefix K/V per step > L2)",
           "fused_append": appended}
    if peaks.get("bf16_tflops_sustained"):
        res["frac_of_measured_bf16_sustained"] = round(tf / peaks["bf16_tflops_sustained"], 4)
        res["frac_of_measured_bf16_burst"] = round(tf / peaks["bf16_tflops"], 4)
    m.release()
    del gathered
    torch.cuda.empty_cache()
    return res


def _time_kernel(fn, flush, iters=20):
    """Median CUDA-event time of `fn` over `iters` launches after 3 warm-ups, L2 flushed before each."""
    times = []
    for i in range(iters + 3):
        if flush is not None:
            flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(100_000)  # keeps the GPU busy while the host enqueues `fn`: no host time in the span
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        if i >= 3:
            times.append(a.elapsed_time(b))
    return statistics.median(times)


def _time_graph(calls, reps: int = 5, min_launches: int = 1) -> float:
    """ms per call of `calls` launched back to back from one CUDA graph (no host time between launches); the
    calls read distinct input copies whose total exceeds the L2, so each reads its input from HBM. Median of
    `reps` replays. With fewer calls than `min_launches` the list is cycled up to that many launches (consecutive
    launches still read different copies): the graph's own start-up latency, which the events around a replay
    include, is then shared by enough launches not to inflate the per-launch time (with two launches per graph
    it added about 2 us to each 50 us launch on a B200)."""
    if len(calls) < min_launches:
        calls = [calls[i % len(calls)] for i in range(min_launches)]
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for fn in calls:
            fn()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for fn in calls:
            fn()
    graph.replay()
    torch.cuda.synchronize()
    times = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b) / len(calls))
    del graph
    return statistics.median(times)


GRAPH_LAUNCHES = 24  # launches per timing graph for the NVFP4 extras


def _copies(nbytes_each: int) -> int:
    return max(2, -(-(320 << 20) // nbytes_each))  # > 2.5x the 126 MB L2 in total


def nvfp4_extras(device, peak):
    """NVFP4 producers at the benchmark shapes (norm T = 4096 / 16384 / 32768 at K = 3072, SiLU T = 4096 / 16384 /
    32768 at K = 12288). `ms`: back-to-back launches from a CUDA graph, each on its own input copy (HBM-resident);
    `ms_single_launch`: one launch between CUDA events after an L2 flush (includes the launch latency). Graphs
    hold at least GRAPH_LAUNCHES launches (the input copies cycled), as the kernels run inside a DiT forward.
    `nvfp4_vs_triton`: the reference's own Triton kernels (fibo/fp4.py:64-116, from the offline install under
    baseline/_ref) timed the same way on the same inputs, next to ours on identical work (no adaLN shift, which
    the reference kernel does not have), with the encodings compared."""
    from types import SimpleNamespace

    from qwenedit_b200.fp4 import global_scale, norm_scale_amax, norm_scale_fp4, silu_mul_amax, silu_mul_fp4

    try:
        from baseline import reference_fp4

        ref = reference_fp4.load()
    except Exception as exc:  # noqa: BLE001
        ref, reference_fp4 = None, None
        ref_missing = f"{type(exc).__name__}: {exc}"
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)  # > L2, rewritten between launches
    out, vs = {}, {}

    def record(name, nbytes, calls, single):
        ms = _time_graph(calls, min_launches=GRAPH_LAUNCHES)
        ms1 = _time_kernel(single, flush)
        out[name] = {"ms": round(ms, 4), "GB/s": round(nbytes / ms / 1e6, 1),
                     "frac_of_measured_hbm": round(nbytes / ms / 1e6 / peak, 4), "ms_single_launch": round(ms1, 4)}

    def versus(name, nbytes, ours_calls, ref_calls, compare):
        if ref is None:
            return
        ours_ms = _time_graph(ours_calls, min_launches=GRAPH_LAUNCHES)
        ref_ms = _time_graph(ref_calls, min_launches=GRAPH_LAUNCHES)
        vs[name] = {"ours_ms": round(ours_ms, 4), "triton_ms": round(ref_ms, 4),
                    "ours_GB/s": round(nbytes / ours_ms / 1e6, 1), "triton_GB/s": round(nbytes / ref_ms / 1e6, 1),
                    "speedup": round(ref_ms / ours_ms, 3), "parity": compare()}

    K = 3072
    norm = SimpleNamespace(weight=(1 + 0.02 * torch.randn(K, device=device)).bfloat16(), eps=1e-6)
    scale = (0.1 * torch.randn(1, K, device=device)).bfloat16()
    shift = (0.1 * torch.randn(1, K, device=device)).bfloat16()
    for T in (4096, 16384, 32768):
        xs = [torch.randn(1, T, K, dtype=torch.bfloat16, device=device) for _ in range(_copies(T * K * 2))]
        gs = global_scale(norm_scale_amax(xs[0], norm, scale, None, None, shift=shift))
        pad = -(-T // 128) * 128
        nbytes = T * K * 2 + K * 2 * 3 + T * K // 2 + pad * K // 16
        record(f"norm_scale_fp4_T{T}", nbytes,
               [lambda x=x: norm_scale_fp4(x, norm, scale, None, None, gs, shift=shift) for x in xs],
               lambda: norm_scale_fp4(xs[0], norm, scale, None, None, gs, shift=shift))
        if T == 32768:  # the calibration pre-pass reads x alone
            record(f"norm_scale_amax_T{T}", T * K * 2 + K * 2 * 3,
                   [lambda x=x: norm_scale_amax(x, norm, scale, None, None, shift=shift) for x in xs],
                   lambda: norm_scale_amax(xs[0], norm, scale, None, None, shift=shift))

        def cmp_norm():
            a = norm_scale_fp4(xs[0], norm, scale, None, None, gs)
            b = ref.norm_scale_fp4(xs[0], norm, scale, None, None, gs)
            st = reference_fp4.compare_nvfp4(a.q, a.sf, b.q, b.sf, gs.item(), T, K)
            return {k: st[k] for k in ("bit_exact", "frac_elements_differing", "max_code_step_same_scale",
                                       "dequant_max_abs_err")}

        versus(f"norm_scale_fp4_T{T}", T * K * 2 + K * 2 * 2 + T * K // 2 + pad * K // 16,
               [lambda x=x: norm_scale_fp4(x, norm, scale, None, None, gs) for x in xs],
               [lambda x=x: ref.norm_scale_fp4(x, norm, scale, None, None, gs) for x in xs], cmp_norm)
        del xs
    K = 12288
    for T in (4096, 16384, 32768):
        n = _copies(2 * T * K * 2)
        gv = [(torch.randn(T, K, dtype=torch.bfloat16, device=device),
               torch.randn(T, K, dtype=torch.bfloat16, device=device)) for _ in range(n)]
        gs = global_scale(silu_mul_amax(gv[0][0], gv[0][1]))
        pad = -(-T // 128) * 128
        nbytes = 2 * T * K * 2 + T * K // 2 + pad * K // 16
        record(f"silu_mul_fp4_T{T}", nbytes, [lambda g=g, v=v: silu_mul_fp4(g, v, gs) for g, v in gv],
               lambda: silu_mul_fp4(gv[0][0], gv[0][1], gs))
        if T == 16384:
            record(f"silu_mul_amax_T{T}", 2 * T * K * 2, [lambda g=g, v=v: silu_mul_amax(g, v) for g, v in gv],
                   lambda: silu_mul_amax(gv[0][0], gv[0][1]))

        def cmp_silu():
            a = silu_mul_fp4(gv[0][0], gv[0][1], gs)
            b = ref.silu_mul_fp4(gv[0][0], gv[0][1], gs)
            st = reference_fp4.compare_nvfp4(a.q, a.sf, b.q, b.sf, gs.item(), T, K)
            return {k: st[k] for k in ("bit_exact", "frac_elements_differing", "max_code_step_same_scale",
                                       "dequant_max_abs_err")}

        versus(f"silu_mul_fp4_T{T}", nbytes, [lambda g=g, v=v: silu_mul_fp4(g, v, gs) for g, v in gv],
               [lambda g=g, v=v: ref.silu_mul_fp4(g, v, gs) for g, v in gv], cmp_silu)
        del gv
    out["nvfp4_vs_triton"] = vs if ref is not None else {"unavailable": ref_missing}
    return out


def nvfp4_cpu(rows_norm: int = 8192, rows_silu: int = 1024):
    """NVFP4 producers on the host cores: the oracle's C restatement of the reference kernels (scalar code,
    one 128-row-aligned chunk of rows per thread). Returns GB/s at the kernels' algorithmic bytes."""
    from concurrent.futures import ThreadPoolExecutor

    from oracle import nvfp4_ref

    lib = nvfp4_ref.lib()
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(0)

    def bf16_bits(shape, scale=1.0, shift=0.0):
        v = torch.from_numpy((rng.standard_normal(shape) * scale + shift).astype(np.float32)).bfloat16()
        return v.view(torch.int16).numpy().view(np.uint16).copy()

    def run(M, K, row_fn):
        chunk = max(128, -(-M // threads) // 128 * 128)
        starts = list(range(0, M, chunk))
        with ThreadPoolExecutor(len(starts)) as ex:
            t0 = time.perf_counter()
            list(ex.map(lambda r0: row_fn(r0, min(chunk, M - r0)), starts))
            return time.perf_counter() - t0, len(starts)

    out = {}
    K = 3072
    x, w = bf16_bits((rows_norm, K)), bf16_bits((K,), 0.02, 1.0)
    mod, sh = bf16_bits((1, K), 0.1), bf16_bits((1, K), 0.1)
    q = np.zeros((rows_norm, K // 2), np.uint8)
    sf = np.zeros((rows_norm, K // 16), np.uint8)
    tile_sf = K // 64 * 512

    def norm_rows(r0, n):
        scratch = np.zeros(2 * 4096, np.float32)
        p = lambda a, off=0: a.ctypes.data + off  # noqa: E731
        lib.ref_norm_scale_fp4(p(x, r0 * K * 2), p(w), p(mod), None, None, p(sh), None, 50.0, n, n, K, 0, 1e-6,
                               p(q, r0 * K // 2), p(sf, r0 // 128 * tile_sf), p(scratch))

    sec, used = run(rows_norm, K, norm_rows)
    nbytes = rows_norm * K * 2 + K * 2 * 3 + rows_norm * K // 2 + rows_norm * K // 16
    out["norm_scale_fp4"] = {"GB/s": round(nbytes / sec / 1e9, 3), "sample": f"x [{rows_norm}, {K}]"}
    K = 12288
    g, v = bf16_bits((rows_silu, K)), bf16_bits((rows_silu, K))
    q = np.zeros((rows_silu, K // 2), np.uint8)
    sf = np.zeros((rows_silu, K // 16), np.uint8)
    tile_sf = K // 64 * 512

    def silu_rows(r0, n):
        scratch = np.zeros(K, np.float32)
        p = lambda a, off=0: a.ctypes.data + off  # noqa: E731
        lib.ref_silu_mul_fp4(p(g, r0 * K * 2), p(v, r0 * K * 2), 50.0, n, K, p(q, r0 * K // 2),
                             p(sf, r0 // 128 * tile_sf), p(scratch))

    sec, used2 = run(rows_silu, K, silu_rows)
    nbytes = 2 * rows_silu * K * 2 + rows_silu * K // 2 + rows_silu * K // 16
    out["silu_mul_fp4"] = {"GB/s": round(nbytes / sec / 1e9, 3), "sample": f"gate, value [{rows_silu}, {K}]"}
    out.update({"cores": max(used, used2), "kind": "port",
                "what": "oracle C restatement of the reference kernels, 128-row chunks across threads"})
    return out


# ---- CPU: the reference's torch ops on the host --------------------------------------------------
def cpu_turns(steps: int, warmup: int, layers: int = CPU_SAMPLE_LAYERS):
    """Turns of the same workload with the oracle pool (index_select / index_copy_ on CPU) over `layers` of
    the 60 layers; returns (GB/s, seconds per turn, threads)."""
    from oracle.pool_ref import RefPagedKVPool

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    tokens = PREFIX + 3 * APPEND + PAGE
    budget = tokens * layers * 2 * ROW
    pool = RefPagedKVPool("dit-cpu", layers, H, D, budget, torch.bfloat16, page_size=PAGE)
    pool.kv.normal_()
    rng = np.random.default_rng(0)
    text = rng.integers(1, 1 << 62, size=TEXT)
    images = [rng.integers(1, 1 << 62, size=IMAGE) for _ in range(steps + warmup + 2)]
    first = np.concatenate([text, images[0]])
    pool.insert(first, pool.alloc(PREFIX), owned_from=0)
    new_kv = torch.randn(layers, 2, APPEND, H, D).bfloat16()
    times = []
    for t in range(warmup + steps):
        t0 = time.perf_counter()
        m = pool.match(np.concatenate([text, images[t]]))
        for _ in range(STEPS_PER_TURN):
            pool.kv.index_select(2, m.indices)  # paged.py:113 (the gather of a scattered prefix)
        slots = pool.alloc(APPEND)
        pool.write(slots, new_kv)
        pool.insert(np.concatenate([text, images[t + 1]]), torch.cat([m.indices[:TEXT], slots]), owned_from=TEXT)
        m.release()
        if t >= warmup:
            times.append(time.perf_counter() - t0)
    sample_bytes = TURN_BYTES * layers / L
    per_turn = statistics.mean(times)
    return sample_bytes / per_turn / 1e9, per_turn, threads


# ---- serving mix: 64 sessions, half 1K and half 2K, hashed to GPUs -------------------------------------
SERVING_SESSIONS = 64
SERVING_ACTIVE = 2  # sessions active at once per GPU: a 2K prefix is 12.5 GB of a 24 GiB pool
IMAGE_TOKENS = {"1k": 4096, "2k": 16384}


def serving_plan(seed: int = 0):
    """Session specs shared by every rank: size, turns (Zipf(1.2) capped at 10), box-edit fraction per turn."""
    rng = np.random.default_rng(seed)
    plan = []
    for i in range(SERVING_SESSIONS):
        turns = int(min(10, rng.zipf(1.2)))
        boxes = [float(rng.uniform(0.1, 0.4)) if rng.random() < 0.2 else 1.0 for _ in range(turns)]
        plan.append({"id": f"session-{i:02d}", "size": "1k" if i % 2 == 0 else "2k", "boxes": boxes})
    return plan


def run_serving(args, rank, world, local):
    """Each rank serves the sessions it owns (stable hash) from its own 24 GiB pool. A turn: match the prefix
    (text + current image); on a full hit, gather it once per denoising step; on a miss (evicted) store the
    recomputed prefix; then append the turn's new image tokens. A box edit recomputes the last `frac` of the
    image tokens (the radix cache can reuse only a prefix), so only those are appended."""
    from qwenedit_b200.paged import PagedKVPool
    from qwenedit_b200.sessions import SessionRouter

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    router = SessionRouter(rank, world)
    plan = [p for p in serving_plan() if router.owns(p["id"])]
    pool = PagedKVPool("dit", L, H, D, POOL_GIB << 30, torch.bfloat16, device, page_size=PAGE)
    pool.index.shuffle_free(2000 + rank)
    stream = torch.cuda.current_stream(device)
    rng = np.random.default_rng(100 + rank)
    new_kv = torch.empty(L, 2, IMAGE_TOKENS["2k"] + TEXT, H, D, dtype=torch.bfloat16, device=device)
    new_kv.normal_()
    outs = {k: torch.empty(L, 2, TEXT + n, H, D, dtype=torch.bfloat16, device=device) for k, n in IMAGE_TOKENS.items()}
    state = {}
    for sp in plan:
        n_img = IMAGE_TOKENS[sp["size"]]
        state[sp["id"]] = {"text": rng.integers(1, 1 << 62, size=TEXT), "image": rng.integers(1, 1 << 62, size=n_img),
                           "turn": 0}
    # SERVING_ACTIVE sessions are active at a time per GPU (the rest queue in a seeded order); requests of the
    # active sessions interleave round-robin, and a finished session hands its slot to the next in the queue
    queue = [plan[i] for i in rng.permutation(len(plan))]
    active, order = [], []
    while queue or active:
        while queue and len(active) < SERVING_ACTIVE:
            active.append(queue.pop(0))
        for sp in list(active):
            t = state[sp["id"]]["turn"]
            order.append((sp, t))
            state[sp["id"]]["turn"] += 1
            if t + 1 >= len(sp["boxes"]):
                active.remove(sp)
    step_events, moved, hits, misses = [], 0, 0, 0
    barrier(world)
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for sp, t in order:
        st = state[sp["id"]]
        vids = np.concatenate([st["text"], st["image"]])
        total = len(vids)
        m = pool.match(vids)
        if m.length == total:
            hits += 1
            out = outs[sp["size"]]
            for _ in range(STEPS_PER_TURN):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                pool.gather_into(m.indices, out)
                b.record(stream)
                step_events.append((a, b))
                moved += 2 * L * 2 * total * ROW
        else:  # evicted (or first turn): the DiT recomputes the uncached tail; store it
            misses += 1
            slots = pool.alloc(total - m.length)
            if slots is not None:
                pool.write(slots, new_kv[:, :, : total - m.length])
                idx = np.concatenate([m.indices._qe_host, slots._qe_host]) if m.length else slots._qe_host
                it = torch.from_numpy(idx.copy())
                it._qe_host = it.numpy()
                pool.insert(vids, it, owned_from=m.length)
                moved += 2 * L * 2 * (total - m.length) * ROW
        m.release()
        # the turn's output becomes the next conditioning image: a box edit changes the last `frac` of it
        frac = sp["boxes"][t]
        n_img = len(st["image"])
        keep = n_img - int(round(frac * n_img)) // PAGE * PAGE
        new_ids = rng.integers(1, 1 << 62, size=n_img - keep)
        st["image"] = np.concatenate([st["image"][:keep], new_ids])
        nv = np.concatenate([st["text"], st["image"]])
        m2 = pool.match(nv)
        slots = pool.alloc(len(nv) - m2.length)
        if slots is not None:
            pool.write(slots, new_kv[:, :, : len(nv) - m2.length])
            idx = np.concatenate([m2.indices._qe_host, slots._qe_host]) if m2.length else slots._qe_host
            it = torch.from_numpy(idx.copy())
            it._qe_host = it.numpy()
            pool.insert(nv, it, owned_from=m2.length)
            moved += 2 * L * 2 * (len(nv) - m2.length) * ROW
        m2.release()
    t1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    elapsed = max_over_ranks(t0.elapsed_time(t1), world, device)
    steps = [a.elapsed_time(b) for a, b in step_events]
    if pool.device_errors():
        raise RuntimeError("a paged copy kernel reported an error")
    total_moved = torch.tensor([float(moved), float(hits), float(misses), float(len(order)),
                                float(pool.usage()["evicted_tokens"])], dtype=torch.float64, device=device)
    all_steps = [steps]
    if world > 1:
        torch.distributed.all_reduce(total_moved)
        gathered = [None] * world
        torch.distributed.all_gather_object(gathered, steps)
        all_steps = gathered
    flat = sorted(x for s_ in all_steps for x in s_)
    pct = (lambda q: flat[min(len(flat) - 1, int(q * len(flat)))]) if flat else (lambda q: None)
    moved_all, hits_all, misses_all, turns_all, evicted_all = [float(v) for v in total_moved.tolist()]
    if rank == 0:
        peak, _ = measured_peak()
        value = moved_all / elapsed / 1e6
        print(json.dumps({
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": int(turns_all),
            "warmup": 0, "ms_per_step": round(elapsed / max(turns_all, 1) * world, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "qwen_image_2.1_serving_64_sessions", "sessions": SERVING_SESSIONS,
                       "sizes": "half 1K (4096+512 prefix), half 2K (16384+512 prefix)",
                       "turns": "Zipf(1.2) capped at 10", "box_edits": "20% of turns, last 10-40% of image tokens",
                       "pool_gib_per_gpu": POOL_GIB, "page_tokens": PAGE, "partition": "stable hash of session id",
                       "active_sessions_per_gpu": SERVING_ACTIVE},
            "frac_of_measured_hbm_per_gpu": round(value / world / peak, 4),
            "step_ms_p50": round(pct(0.5), 4) if flat else None, "step_ms_p99": round(pct(0.99), 4) if flat else None,
            "turns": int(turns_all), "prefix_hits": int(hits_all), "prefix_misses": int(misses_all),
            "evicted_tokens": int(evicted_all), "gpu_launches": len(flat) + 2 * int(turns_all),
        }), flush=True)


# ---- one 2K session head-sharded over all ranks (strong scaling) ---------------------------------------
NVLINK_GBS = 770.0  # measured peer copy per direction per GPU on this node type


def run_headshard(args, rank, world, local):
    """One 2K edit session whose pool is split by head over the ranks (HeadShardedKVPool): every denoising
    step each rank gathers its heads of the 16,896-token prefix locally; once per turn the 16,384 new image
    tokens, held sequence-parallel (rank r has tokens [r T/n, (r+1) T/n) with all heads), are appended with
    the fused head-scatter kernel over NVLink, followed by the stream-ordered barrier."""
    from qwenedit_b200.sharded import HeadShardedKVPool

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    img = IMAGE_TOKENS["2k"]
    prefix = TEXT + img
    pool = HeadShardedKVPool("dit-2k", L, H, D, POOL_GIB << 30, torch.bfloat16, device, page_size=PAGE)
    pool.pool.index.shuffle_free(5)  # same seed on every rank: the index is replicated
    hl = pool.heads_local
    rng = np.random.default_rng(9)  # the session's ids: the same on every rank
    text = rng.integers(1, 1 << 62, size=TEXT)
    images = [rng.integers(1, 1 << 62, size=img) for _ in range(args.steps + args.warmup + 2)]
    lo, hi = rank * img // world, (rank + 1) * img // world
    new_kv = torch.empty(L, 2, hi - lo, H, D, dtype=torch.bfloat16, device=device)
    new_kv.normal_()
    out = torch.empty(L, 2, prefix, hl, D, dtype=torch.bfloat16, device=device)
    first = pool.alloc(prefix)  # turn 0's prefix, computed on a miss: every rank writes its heads
    pool.write(first, torch.randn(L, 2, prefix, hl, D, dtype=torch.bfloat16, device=device))
    pool.insert(np.concatenate([text, images[0]]), first, owned_from=0)
    stream = torch.cuda.current_stream(device)

    def turn(t, ev=None):
        m = pool.match(np.concatenate([text, images[t]]))
        if m.length != prefix:
            raise RuntimeError(f"turn {t}: expected a full prefix hit, got {m.length}")
        for _ in range(STEPS_PER_TURN):
            pool.gather_into(m.indices, out)
        slots = pool.alloc(img)
        if slots is None:
            raise RuntimeError("pool exhausted")
        if ev is not None:
            ev[0].record(stream)
        pool.write_scatter(slots[lo:hi], new_kv)
        if ev is not None:
            ev[1].record(stream)
        pool.barrier()
        idx_host = np.concatenate([m.indices._qe_host[:TEXT], slots._qe_host])
        idx = torch.from_numpy(idx_host)
        idx._qe_host = idx_host
        pool.insert(np.concatenate([text, images[t + 1]]), idx, owned_from=TEXT)
        m.release()

    for t in range(args.warmup):
        turn(t)
    pool.verify_replicas()
    scatter_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(args.steps)]
    barrier(world)
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(args.steps):
        turn(args.warmup + i, scatter_ev[i])
    t1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    elapsed = max_over_ranks(t0.elapsed_time(t1), world, device)
    scatter_ms = max_over_ranks(statistics.mean(a.elapsed_time(b) for a, b in scatter_ev), world, device)
    if pool.device_errors():
        raise RuntimeError("a paged copy kernel reported an error")
    pool.verify_replicas()
    gather_bytes = 2 * L * 2 * prefix * ROW  # all heads, summed over the ranks
    append_bytes = 2 * L * 2 * img * ROW
    turn_bytes = STEPS_PER_TURN * gather_bytes + append_bytes
    nvlink_per_rank = (world - 1) * L * 2 * (hi - lo) * hl * D * 2
    if rank == 0:
        peak, _ = measured_peak()
        value = turn_bytes / (elapsed / args.steps) / 1e6
        print(json.dumps({
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(elapsed / args.steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "qwen_image_2.1_2k_edit_head_sharded", "layers": L, "heads": H, "head_dim": D,
                       "heads_per_gpu": hl, "prefix_tokens": prefix, "append_tokens": img, "page_tokens": PAGE,
                       "gathers_per_turn": STEPS_PER_TURN, "pool_gib_per_gpu": POOL_GIB,
                       "append": "sequence-parallel rows scattered to head owners (qe_append_scatter)"},
            "frac_of_measured_hbm_per_gpu": round(value / world / peak, 4),
            "dit_step_ms_2k": round((elapsed / args.steps - scatter_ms) / STEPS_PER_TURN, 4),
            "scatter": {"ms": round(scatter_ms, 4), "nvlink_bytes_per_gpu": nvlink_per_rank,
                        "nvlink_GB/s_per_gpu": round(nvlink_per_rank / scatter_ms / 1e6, 1) if world > 1 else None,
                        "frac_of_nvlink": round(nvlink_per_rank / scatter_ms / 1e6 / NVLINK_GBS, 4)
                        if world > 1 else None},
            "gpu_launches": args.steps * (STEPS_PER_TURN + 1),
        }), flush=True)
    pool.close()


def profile_case(kind: str) -> None:
    """A small case of one kernel for ncu captures: inputs > L2, a few GB on the device, 6 launches."""
    from types import SimpleNamespace

    from qwenedit_b200.fp4 import norm_scale_fp4, silu_mul_fp4
    from qwenedit_b200.paged import PagedKVPool

    device = torch.device("cuda", 0)
    layers = CPU_SAMPLE_LAYERS  # 8 of the 60 layers: 453 MB read + 453 MB written per gather
    times = []
    if kind in ("gather", "append"):
        pool = PagedKVPool("dit", layers, H, D, (PREFIX + APPEND + PAGE) * layers * 2 * ROW, torch.bfloat16, device,
                           page_size=PAGE)
        pool.index.shuffle_free(5)
        pool.kv.normal_()
        n = PREFIX if kind == "gather" else APPEND
        slots = pool.alloc(n)
        buf = torch.randn(layers, 2, n, H, D, device=device).bfloat16()
        fn = (lambda: pool.gather_into(slots, buf)) if kind == "gather" else (lambda: pool.write(slots, buf))
    elif kind == "short_rows":  # 768 B rows (3 of 24 heads: an 8-way head-sharded pool), 60 layers, 2K prefix
        hl, n = 3, 16896
        pool = PagedKVPool("dit-shard", L, hl, D, 24 << 30, torch.bfloat16, device, page_size=PAGE)
        pool.index.shuffle_free(5)
        slots = pool.alloc(n)
        buf = torch.empty(L, 2, n, hl, D, dtype=torch.bfloat16, device=device)
        fn = lambda: pool.gather_into(slots, buf)  # noqa: E731
    elif kind == "attention":  # one layer of the 1K edit's joint attention (4096 queries, 4608 + 4096 keys, 24 heads)
        from qwenedit_b200.attention import PagedPrefix, paged_attention

        pool = PagedKVPool("dit", 1, H, D, (PREFIX + 2 * PAGE) * 2 * ROW, torch.bfloat16, device, page_size=PAGE)
        pool.index.shuffle_free(5)
        pool.kv.normal_()
        prefix = PagedPrefix(pool, pool.alloc(PREFIX))
        q, k_own, v_own = (torch.randn(IMAGE, H, D, device=device).bfloat16() for _ in range(3))
        out = torch.empty_like(q)
        fn = lambda: paged_attention(q, prefix, 0, k_own, v_own, out=out)  # noqa: E731
    elif kind == "gather_heads":  # the encoder's partial hit: 28 layers x 4 heads, 4096 prefix tokens head-major
        pool = PagedKVPool("encoder", 28, 4, D, 8192 * 28 * 2 * 4 * D * 2, torch.bfloat16, device)
        pool.index.shuffle_free(5)
        pool.kv.normal_()
        slots = pool.alloc(4096)
        fn = lambda: pool.gather_heads(slots, 4096 + 256)  # noqa: E731
    elif kind == "mask_blend":  # per-step latent blend on 16 x 16384 x 64 bf16 latents (inputs > L2 in total)
        from qwenedit_b200.latents import mask_blend

        lat = torch.randn(16, 16384, 64, device=device).bfloat16()
        x0, eps = torch.randn_like(lat), torch.randn_like(lat)
        msk = torch.rand(16, 16384, 1, device=device)
        sigma = torch.tensor(0.5, device=device)
        fn = lambda: mask_blend(lat, x0, eps, msk, sigma)  # noqa: E731
    elif kind in ("norm_amax", "silu_amax"):
        from qwenedit_b200.fp4 import norm_scale_amax, silu_mul_amax

        if kind == "norm_amax":
            x = torch.randn(1, 32768, 3072, dtype=torch.bfloat16, device=device)
            norm = SimpleNamespace(weight=torch.ones(3072, dtype=torch.bfloat16, device=device), eps=1e-6)
            sc = (0.1 * torch.randn(1, 3072, device=device)).bfloat16()
            fn = lambda: norm_scale_amax(x, norm, sc, None, None, shift=sc)  # noqa: E731
        else:
            g = torch.randn(4096, 12288, dtype=torch.bfloat16, device=device)
            v = torch.randn(4096, 12288, dtype=torch.bfloat16, device=device)
            fn = lambda: silu_mul_amax(g, v)  # noqa: E731
    elif kind == "norm":
        T, K = 32768, 3072
        x = torch.randn(1, T, K, dtype=torch.bfloat16, device=device)
        norm = SimpleNamespace(weight=torch.ones(K, dtype=torch.bfloat16, device=device), eps=1e-6)
        sc = (0.1 * torch.randn(1, K, device=device)).bfloat16()
        gs = torch.tensor([50.0], device=device)
        fn = lambda: norm_scale_fp4(x, norm, sc, None, None, gs, shift=sc)  # noqa: E731
    else:
        T, K = 4096, 12288
        g = torch.randn(T, K, dtype=torch.bfloat16, device=device)
        v = torch.randn(T, K, dtype=torch.bfloat16, device=device)
        gs = torch.tensor([50.0], device=device)
        fn = lambda: silu_mul_fp4(g, v, gs)  # noqa: E731
    for i in range(6):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        if i >= 3:
            times.append(a.elapsed_time(b))
    print(json.dumps({"profile_case": kind, "ms": [round(t, 4) for t in times]}), flush=True)


def main():
    args = parse()
    if args.profile:
        profile_case(args.profile)
        return
    rank, world, local = dist_setup(args) if args.impl == "ours" else (
        int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0)))
    if args.impl == "reference":
        if rank != 0:
            return
        gbs, per_turn, threads = cpu_turns(args.steps, args.warmup)
        sample = (f"{CPU_SAMPLE_LAYERS} of {L} layers per turn (same per-layer shapes; the cost is linear in "
                  f"layers); {args.steps} timed turns after {args.warmup} warm-up")
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_turn * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": dict(CONFIG, layers_run=CPU_SAMPLE_LAYERS,
                           step="one turn over the sampled layers: 8 prefix gathers + 1 append"),
            "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }), flush=True)
        return

    if args.workload in ("serving", "headshard"):
        (run_serving if args.workload == "serving" else run_headshard)(args, rank, world, local)
        if world > 1:
            torch.distributed.destroy_process_group()
        return
    r = run_ours(args, rank, world, local)
    peak, peak_src = measured_peak()
    value = TURN_BYTES * world / (r["elapsed_ms"] / args.steps) / 1e6  # GB/s over all ranks
    achieved = GATHER_BYTES / r["avg_gather_ms"] / 1e6
    traffic = committed_traffic("paged_gather_pages")
    e2e = TURN_BYTES * world / (r["e2e_ms"] / args.steps) / 1e6
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gbs, per_turn, threads = cpu_turns(steps=6, warmup=1)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": f"6 turns (+1 warm-up) over {CPU_SAMPLE_LAYERS} of {L} layers; reference torch ops "
                         "(index_select / index_copy_) + restated prefix index",
               "ms_per_sample_turn": round(per_turn * 1e3, 3)}
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(r["elapsed_ms"] / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": CONFIG,
            "dit_step_ms_1k": round(r["avg_gather_ms"], 4),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4),
                         "traffic": None if traffic is None else traffic["read"] + traffic["write"],
                         "traffic_read": None if traffic is None else traffic["read"],
                         "traffic_write_lower_bound": None if traffic is None else traffic["write"],
                         "traffic_source": "ncu, full 60-layer launch (profiles/small_kernels.md)",
                         "kernel": "paged_gather (block table)",
                         "peak_source": peak_src,
                         "algorithmic_bytes_per_launch": GATHER_BYTES},
            "frac_of_measured_hbm": round(value / world / peak, 4),
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e, 1), "unit": "GB/s", "h2d_bytes_per_step": int(r["h2d"]),
                    "d2h_bytes_per_step": int(r["d2h"])},
            "gpu_launches": args.steps * (STEPS_PER_TURN + 1),
            "clocks": r["clocks"],
            "extras": r["extras"],
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
