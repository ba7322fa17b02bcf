"""Benchmark of the per-chunk causal self-attention hot path (704x1280, 12-chunk KV).

One step = one chunk of the streaming rollout through the 30-layer attention
stack, as the reference's compressed pipeline runs it
(pipeline/causal_diffusion_inference_compressed.py:621-734 with the shipped
4-step DMD config): 4 denoising forwards + 1 clean-KV forward, each writing the
chunk's roped K/V into every layer's cache and attending the chunk's 2640
queries over the cache (1 sink + 5 recent + 6 retrieved landmarks = 31680 keys)
plus the chunk itself (34320 keys), then the landmark-bank update: admission
with eviction, pose top-k retrieval from the 30-entry bank and the gather of
sink | recent | landmarks into all 30 layers' caches.

value = attention FLOPs of the step (5 x 30 x 4*Lq*Lk*H*D) / step time, whole
job.  With --gpus N > 1 the step runs Ulysses head-parallel (H/N heads per
rank, head-resident caches and bank; the sequence-sharded q/k/v and the output
are exchanged by this package's peer-memory scatter kernels, the RoPE and cache
write fused into the inbound one), strong scaling.

--impl reference times the reference's own CPU attention path (torch SDPA on
the host cores, the branch wan_5b/modules/attention.py:164-179 takes without
flash-attention) on a bounded sample of the same workload.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from reworld_b200.landmark import budget_split  # noqa: E402

# workload: 704x1280 video, latent 44x80, 2x2 patches -> 22x40 tokens per frame, 3 frames per chunk
FRAMES, TOK_H, TOK_W = 3, 22, 40
CT = FRAMES * TOK_H * TOK_W                  # 2640 query tokens per chunk
N_LAYERS, HEADS, HEAD_DIM = 30, 24, 128
# the kv_compression knobs of the shipped v15b run (--kv_budget_chunks 12 --kv_n_sink 1 --kv_recent_w 5,
# bank of 30); the pipeline's budget split turns them into sink 1 + recent 5 + 6 landmarks
BUDGET_CHUNKS, SINK_KNOB, RECENT_CAP, LANDMARK_K, POLICY = 12, 1, 5, 30, "v15b"
SPLIT = budget_split(BUDGET_CHUNKS, SINK_KNOB, RECENT_CAP, LANDMARK_K, POLICY,
                     cache_tokens=(BUDGET_CHUNKS + 1) * CT, chunk_tokens=CT)
N_SINK, RECENT_W, N_LANDMARK, BANK_K = SPLIT.n_sink, SPLIT.recent_w, SPLIT.n_landmark, SPLIT.K
BUDGET = SPLIT.budget                        # 12 chunks
LK = (BUDGET + 1) * CT                       # 34320 keys (cache + the chunk itself)
FORWARDS_PER_CHUNK = 5                       # 4 denoise + 1 clean-KV forward
REVISIT_EVERY = 8                            # chunks between returns to an earlier place
METRIC = "causal chunk-attn TFLOP/s + ms/chunk, 704x1280 12-chunk KV, 1/2/4/8 B200"
WORKLOAD = ("704x1280 chunk (3 latent frames, 2640 tokens) x 30 layers x 24 heads x 128, KV budget 12 chunks "
            "(1 sink + 5 recent + 6 landmarks = 31680 keys) + the chunk itself = 34320 keys; 5 forwards/chunk "
            "(4 denoise + 1 clean-KV); bank of 30 with pose top-6 retrieval and all-layer gather per chunk")


def attn_flops(lq, lk, h):
    return 4.0 * lq * lk * h * HEAD_DIM


class Clocks:
    """Samples nvidia-smi every 50 ms during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.skip = 0
        self.path = tempfile.mktemp(suffix=".csv")

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=self.fh, stderr=subprocess.DEVNULL)
            # the timed region starts only once the sampler is producing lines
            t0 = time.time()
            while time.time() - t0 < 5.0:
                self.fh.flush()
                if os.path.getsize(self.path) > 0:
                    break
                time.sleep(0.02)
            time.sleep(0.06)
            self.skip = sum(1 for _ in open(self.path))   # lines sampled before the timed region
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.fh.close()

    def summary(self):
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for i, line in enumerate(open(self.path)):
            if i < self.skip:
                continue
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows),
                "power_w_max": max((float(r[3]) for r in rows if r[3].replace(".", "").isdigit()), default=None)}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("bf16_tflops", 1590.0), d.get("bf16_tflops_sustained", 1400.0), d.get("hbm_gbs", 6650.0), \
            "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


def profiled_traffic():
    """DRAM bytes per attention launch from the committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", "attn_pair_kernel_2640x34320.txt")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("traffic_bytes_per_launch_full_size:"):
            try:
                return float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


# ------------------------------------------------------------------ GPU arm
class Rollout:
    """Device state of the rollout on one rank: per-layer caches for this rank's
    heads, the landmark bank stack, the chunk inputs."""

    def __init__(self, device, heads, seq_shard, world, rank, group):
        from reworld_b200 import RopeArgs, build_freqs, device_table
        from reworld_b200.poses import random_walk
        self.dev, self.H, self.world, self.rank, self.group = device, heads, world, rank, group
        self.cap = (BUDGET + 1) * CT
        g = torch.Generator(device=device).manual_seed(1234 + rank)
        self.sp = None
        if world > 1:
            # head-resident caches in symmetric memory: peers write the chunk's roped K/V into them
            from reworld_b200.ulysses import UlyssesP2P
            self.sp = UlyssesP2P(group, N_LAYERS, self.cap, CT, HEADS, HEAD_DIM, device=device)
            self.cache_k = [self.sp.cache_k(l) for l in range(N_LAYERS)]
            self.cache_v = [self.sp.cache_v(l) for l in range(N_LAYERS)]
        else:
            self.cache_k = [torch.zeros(1, self.cap, heads, HEAD_DIM, dtype=torch.bfloat16, device=device)
                            for _ in range(N_LAYERS)]
            self.cache_v = [torch.zeros_like(c) for c in self.cache_k]
        # activations of the chunk per layer: sequence-sharded when world > 1
        shape = (1, seq_shard, HEADS, HEAD_DIM)
        self.q = [torch.randn(shape, generator=g, device=device).to(torch.bfloat16) for _ in range(N_LAYERS)]
        self.k = [torch.randn(shape, generator=g, device=device).to(torch.bfloat16) for _ in range(N_LAYERS)]
        self.v = [torch.randn(shape, generator=g, device=device).to(torch.bfloat16) for _ in range(N_LAYERS)]
        self.out = [torch.empty(1, CT, heads, HEAD_DIM, dtype=torch.bfloat16, device=device) for _ in range(N_LAYERS)]
        self.bank = None
        self.new_bank()
        self.table = device_table(build_freqs(HEAD_DIM, 12 / 22, 20 / 40), device)
        self.RopeArgs = RopeArgs
        # camera context of every frame (the model's prope_context), on the device as in the
        # pipeline; the bank's pose of a chunk is chunk_pose over its frames
        frames = random_walk(512 * FRAMES, seed=0, step_t=0.1 / FRAMES, step_deg=5.0 / FRAMES,
                             revisit_every=REVISIT_EVERY * FRAMES)
        self.frame_ctx = torch.from_numpy(np.stack(frames)).to(device).unsqueeze(0)
        self.frame_ctx_host = self.frame_ctx.cpu()   # the camera path is host input: poses need no device read
        self._pose = None
        self.launches = 0
        self.flops_all = 0.0          # attention FLOPs of all heads issued so far (whole job)
        self.host_issue_s = []        # host time to enqueue each forward (30 layers of launches)
        self.scatter_events = []      # Ulysses: event pairs around each layer's q/k/v scatter
        self._split_cache = {}
        self.attn_events = []
        self.step_marks = []          # per timed step: events at each forward's start, the bank update's start and end
        self.bank_host_s = []         # host time of each bank update (its decision is read back to the host)

    def new_bank(self):
        """A cold bank (budget split of the v15b knobs) and an empty cache."""
        from reworld_b200.landmark import LandmarkBankStack
        self.bank = None
        self._pose = None
        torch.cuda.empty_cache()
        self.bank = LandmarkBankStack.from_budget(CT, N_LAYERS, self.H, HEAD_DIM, BUDGET_CHUNKS, SINK_KNOB,
                                                  RECENT_CAP, LANDMARK_K, POLICY, cache_tokens=self.cap,
                                                  device=self.dev)
        self.chunk = 0
        self.tot = 0

    def fill_bank(self, n_chunks):
        """Cold-start the cache: run the bank update for n_chunks (no attention)."""
        for _ in range(n_chunks):
            for l in range(N_LAYERS):
                self.cache_k[l][:, self.tot:self.tot + CT].normal_()
                self.cache_v[l][:, self.tot:self.tot + CT].normal_()
            self.bank_update()

    def prepare_bank(self):
        """The chunk's pose and its bank decision, queued before the chunk's forwards
        (the decision depends on poses only), so the update after them does not wait
        for the device to drain."""
        from reworld_b200.landmark import chunk_pose
        c = self.chunk
        self._pose = chunk_pose(self.frame_ctx_host[:, :(c + 1) * FRAMES], FRAMES)
        self.bank.prepare(self._pose, self._pose)

    def bank_update(self):
        from reworld_b200.landmark import chunk_pose
        c = self.chunk
        pose = self._pose if self._pose is not None else chunk_pose(self.frame_ctx_host[:, :(c + 1) * FRAMES], FRAMES)
        self._pose = None
        src_k = [ck[0, self.tot:self.tot + CT] for ck in self.cache_k]
        src_v = [cv[0, self.tot:self.tot + CT] for cv in self.cache_v]
        R = self.bank.add_chunk_from(src_k, src_v, pose, pose)
        self.tot = self.bank.write_into_caches(self.cache_k, self.cache_v, R)
        self.launches += 3        # pack copy, bank decision, gather
        self.chunk += 1

    def forward(self, time_attn=False):
        from reworld_b200 import chunk_attention, rope_kv_store
        start_frame = (self.chunk * CT) // (TOK_H * TOK_W)
        rope = self.RopeArgs(self.table, (FRAMES, TOK_H, TOK_W), start_frame % 1000)
        for l in range(N_LAYERS):
            q, k, v = self.q[l], self.k[l], self.v[l]
            lk = self.tot + CT
            self.flops_all += attn_flops(CT, lk, HEADS)
            if self.sp is not None:
                # peer-memory exchange: the q/k/v scatter (RoPE + cache write fused; signals the
                # ranks when done) and the attention on the local heads (waits for every rank's
                # scatter, stores each output row at its owner rank, signals when done); nothing
                # reads the outputs inside the step, so no wait for them
                ev = sev = None
                if time_attn:
                    ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                    sev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                self.sp.layer(l, q, k, v, self.tot, rope=rope, attn_events=ev, sync_output=False, scatter_events=sev)
                if time_attn:
                    self.attn_events.append((ev[0], ev[1], lk))
                    self.scatter_events.append(sev)
                self.launches += 2 + (1 if self._split(lk) else 0)   # scatter, attention (+ merge)
                continue
            rope_kv_store(k, v, self.cache_k[l], self.cache_v[l], self.tot, rope=rope)
            if time_attn:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
            o = chunk_attention(q, self.cache_k[l][:, :lk], self.cache_v[l][:, :lk], rope=rope, out=self.out[l])
            if time_attn:
                e1.record()
                self.attn_events.append((e0, e1, lk))
            self.launches += 2 + (1 if self._split(lk) else 0)   # store, attention (+ key-split combine)

    def _split(self, lk):
        from reworld_b200 import _native
        key = lk
        if key not in self._split_cache:
            self._split_cache[key] = _native.lib().rw_attn_workspace_bytes(1, CT, lk, self.H) > 0
        return self._split_cache[key]

    def step(self, time_attn=False):
        marks = [] if time_attn else None
        self.prepare_bank()
        for i in range(FORWARDS_PER_CHUNK):
            t0 = time.perf_counter()
            if marks is not None:
                marks.append(torch.cuda.Event(enable_timing=True))
                marks[-1].record()
            # per-launch events only in the first forward: an event between two kernels
            # keeps the second from starting early (programmatic dependent launch)
            self.forward(time_attn and i == 0)
            self.host_issue_s.append(time.perf_counter() - t0)
        if marks is not None:
            marks.append(torch.cuda.Event(enable_timing=True))
            marks[-1].record()
        t0 = time.perf_counter()
        self.bank_update()
        if marks is not None:
            self.bank_host_s.append(time.perf_counter() - t0)
            marks.append(torch.cuda.Event(enable_timing=True))
            marks[-1].record()
            self.step_marks.append(marks)


def run_gpu(args):
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        group = dist.group.WORLD
    from reworld_b200 import _native
    heads = HEADS // world
    seq_shard = CT // world
    ro = Rollout(dev, heads, seq_shard, world, rank, group)
    ro.fill_bank(BUDGET + BANK_K + 2)          # steady state: bank full, 12-chunk cache
    for _ in range(args.warmup):
        ro.step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    launches0 = ro.launches
    ro.attn_events.clear()
    ro.host_issue_s.clear()
    ro.scatter_events.clear()
    ro.step_marks.clear()
    ro.bank_host_s.clear()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("timed_steps")
        e0.record()
        for _ in range(args.steps):
            ro.step(time_attn=True)
        e1.record()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    if world > 1:
        dist.barrier()
    ms = e0.elapsed_time(e1) / args.steps
    host_issue_ms = 1e3 * statistics.median(ro.host_issue_s)
    launches = (ro.launches - launches0) // args.steps
    attn_ms = [a.elapsed_time(b) for a, b, _ in ro.attn_events]
    attn_lk = [lk for _, _, lk in ro.attn_events]
    _native.check_status(dev)
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())

    # where a step's time goes (device clock on this rank): the forwards and the bank update
    fwd_ms = [m[i].elapsed_time(m[i + 1]) for m in ro.step_marks for i in range(FORWARDS_PER_CHUNK)]
    bank_ms = [m[-2].elapsed_time(m[-1]) for m in ro.step_marks]
    breakdown = {"forward_ms": round(statistics.median(fwd_ms), 3),
                 "layer_us": round(1e3 * statistics.median(fwd_ms) / N_LAYERS, 1),
                 "attention_us": round(1e3 * statistics.median(a.elapsed_time(b) for a, b, _ in ro.attn_events), 1),
                 "bank_update_ms": round(statistics.median(bank_ms), 3),
                 "bank_update_host_ms": round(1e3 * statistics.median(ro.bank_host_s), 3),
                 "note": "medians over the timed steps on rank 0; a layer = " +
                         ("scatter + attention (+ merge) + launch gaps" if world > 1 else
                          "RoPE store + attention (+ merge)") +
                         "; bank update = pack of the chunk, gather of all layers' caches (its decision was "
                         "queued before the forwards and is read back without draining the device)"}
    exchange = None
    if world > 1:
        # the seq->head exchange of one layer: bytes this rank's scatter sends over NVLink
        # (the other ranks' heads of its q, k, v rows) over the scatter kernel's time
        sc_ms = statistics.median(a.elapsed_time(b) for a, b in ro.scatter_events)
        nv_bytes = 3 * seq_shard * HEADS * HEAD_DIM * 2 * (world - 1) // world
        out_bytes = CT * heads * HEAD_DIM * 2 * (world - 1) // world
        exchange = {"scatter_us": round(sc_ms * 1e3, 2), "scatter_nvlink_bytes_per_gpu": nv_bytes,
                    "scatter_gbs_per_gpu": round(nv_bytes / (sc_ms * 1e-3) / 1e9, 1),
                    "nvlink_peak_gbs_per_direction": 900.0, "measured_peer_copy_gbs": 770.0,
                    "frac_of_nominal": round(nv_bytes / (sc_ms * 1e-3) / 1e9 / 900.0, 4),
                    "output_nvlink_bytes_per_gpu": out_bytes,
                    "output_exchange": "stored by the attention epilogue straight into the owner ranks' buffers "
                                       "(overlapped with the remaining tiles' compute; no kernel of its own)",
                    "note": "the scatter also applies k's RoPE and writes the caches; per layer, median over "
                            "the timed steps"}
    # e2e: host buffers through the public API, copies inside the timed region
    e2e = run_e2e(ro, args, dev) if world == 1 else run_e2e_sp(ro, args, dev)
    parity = sp_parity(ro, dev, world, rank, group) if world > 1 else None
    stress_sp = stress_sp_measure(dev, world, rank, group) if world > 1 else None
    seq_kv = seq_kv_sp_measure(dev, world, rank, group) if world > 1 else None

    step_flops = FORWARDS_PER_CHUNK * N_LAYERS * attn_flops(CT, LK, HEADS)
    attn_avg_ms = sum(attn_ms) / len(attn_ms)
    per_launch_flops = attn_flops(CT, statistics.mean(attn_lk), heads)
    burst, sustained, hbm, peak_src = load_peaks()
    achieved = per_launch_flops / (attn_avg_ms * 1e-3) / 1e12
    traffic = profiled_traffic()
    if traffic is not None and heads != HEADS:
        # the capture is of the 24-head launch; a rank's launch covers heads / 24 of its
        # units (DRAM bytes grow with the heads: q, o and every head's K/V rows)
        traffic = round(traffic * heads / HEADS)
    extra = {}
    if rank == 0 and world == 1:
        extra = gpu_side_baselines(ro, dev)
    cold = rollout_cold(ro, dev, world, group, n_chunks=32)
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(step_flops / (ms_max * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max, 3),
            "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded N(0,1) activations, random-walk camera poses)",
            "config": {"workload": WORKLOAD, "step": "one chunk: 5 forwards x 30 layers + bank update + gather",
                       "Lq": CT, "Lk": LK, "layers": N_LAYERS, "heads": HEADS, "head_dim": HEAD_DIM,
                       "parallelism": f"ulysses{world}" if world > 1 else "single",
                       "l2": "inputs larger than L2 (12.5 GB of caches + 1.5 GB activations per step)"},
            "ms_per_forward": round(ms_max / FORWARDS_PER_CHUNK, 3),
            "host_issue_ms_per_forward": round(host_issue_ms, 3),
            "chunks_per_s": round(1000.0 / ms_max, 3),
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1),
                         "peak": sustained, "unit": "TFLOP/s", "frac": round(achieved / sustained, 4),
                         "peak_kind": f"bf16 sustained ({peak_src}); burst {burst}",
                         "frac_of_burst": round(achieved / burst, 4),
                         "kernel": "rw_attn_fwd", "avg_launch_ms": round(attn_avg_ms, 4),
                         "flops_per_launch": per_launch_flops, "traffic": traffic,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of the 24-head launch"
                                           + (f", scaled by {heads}/{HEADS} heads" if heads != HEADS else "")},
            "gpu_launches": launches * args.steps,
            "clocks": clk.summary(),
        }
        if e2e is not None:
            line["e2e"] = e2e
        if parity is not None:
            line["sp_parity"] = parity
        if stress_sp is not None:
            line["stress_b4_sp"] = stress_sp
        if seq_kv is not None:
            line["seq_sharded_kv_sp"] = seq_kv
        line["step_breakdown"] = breakdown
        if exchange is not None:
            line["exchange"] = exchange
            breakdown["scatter_us"] = exchange["scatter_us"]
        line["rollout_cold32"] = cold
        line.update(extra)
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(budget_s=args.cpu_seconds)
        print(json.dumps(line), flush=True)
    if world > 1:
        ro.sp.finish()                 # every rank's last output rows have landed (no peer still writes here)
        torch.cuda.synchronize()
        dist.barrier()
        ro = None                      # release the symmetric buffers before the group goes away
        dist.barrier()
        dist.destroy_process_group()


def run_e2e(ro, args, dev):
    """Same chunk step through the public API with q/k/v of every forward coming
    from pinned host memory and every layer's output copied back to pinned host
    memory; copies run on side streams overlapped with the compute stream."""
    from reworld_b200 import chunk_attention, rope_kv_store
    comp = torch.cuda.current_stream(dev)
    h2d = torch.cuda.Stream(dev)
    d2h = torch.cuda.Stream(dev)
    shape = (1, CT, HEADS, HEAD_DIM)
    host_in = [torch.randn(3, *shape).to(torch.bfloat16).pin_memory() for _ in range(2)]
    host_out = [torch.empty(shape, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    dev_in = [torch.empty((3, *shape), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    dev_out = [torch.empty(shape, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_used = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    ev_read = [torch.cuda.Event() for _ in range(2)]
    for e in ev_used + ev_read:
        e.record(comp)
    bytes_in = 3 * CT * HEADS * HEAD_DIM * 2
    bytes_out = CT * HEADS * HEAD_DIM * 2

    def step():
        n = 0
        ro.prepare_bank()
        for _f in range(FORWARDS_PER_CHUNK):
            start_frame = (ro.chunk * CT) // (TOK_H * TOK_W)
            rope = ro.RopeArgs(ro.table, (FRAMES, TOK_H, TOK_W), start_frame % 1000)
            for l in range(N_LAYERS):
                b = n & 1
                with torch.cuda.stream(h2d):
                    h2d.wait_event(ev_used[b])
                    dev_in[b].copy_(host_in[b], non_blocking=True)
                    ev_in[b].record(h2d)
                comp.wait_event(ev_in[b])
                comp.wait_event(ev_read[b])
                q, k, v = dev_in[b][0], dev_in[b][1], dev_in[b][2]
                rope_kv_store(k, v, ro.cache_k[l], ro.cache_v[l], ro.tot, rope=rope)
                lk = ro.tot + CT
                chunk_attention(q, ro.cache_k[l][:, :lk], ro.cache_v[l][:, :lk], rope=rope, out=dev_out[b])
                ev_used[b].record(comp)
                ev_out[b].record(comp)
                with torch.cuda.stream(d2h):
                    d2h.wait_event(ev_out[b])
                    host_out[b].copy_(dev_out[b], non_blocking=True)
                    ev_read[b].record(d2h)
                n += 1
        ro.bank_update()

    for _ in range(max(1, args.warmup // 2)):
        step()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(comp)
    for _ in range(args.steps):
        step()
    comp.wait_stream(d2h)
    t1.record(comp)
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / args.steps
    step_flops = FORWARDS_PER_CHUNK * N_LAYERS * attn_flops(CT, LK, HEADS)
    n_io = FORWARDS_PER_CHUNK * N_LAYERS
    return {"value": round(step_flops / (ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s", "ms_per_step": round(ms, 3),
            "h2d_bytes_per_step": n_io * bytes_in, "d2h_bytes_per_step": n_io * bytes_out,
            "path": "reworld_b200.rope_kv_store + chunk_attention with pinned host q/k/v in, output out, "
                    "copies on side streams overlapped with compute"}


def rollout_cold(ro, dev, world, group, n_chunks=32):
    """The streaming rollout from a cold cache: a new bank, then n_chunks chunks
    (5 forwards x 30 layers each, attention over the cache as it fills, bank
    update, a return to an earlier place every 8 chunks), timed as one region
    with CUDA events (max over ranks)."""
    import torch.distributed as dist
    ro.new_bank()
    f0 = ro.flops_all
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier(group)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(n_chunks):
        ro.step()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b)], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    ms = float(t.item())
    fl = ro.flops_all - f0
    return {"chunks": n_chunks, "ms": round(ms, 2), "chunks_per_s": round(n_chunks / (ms * 1e-3), 3),
            "ms_per_chunk": round(ms / n_chunks, 3), "attn_tflops": round(fl / (ms * 1e-3) / 1e12, 1),
            "n_gpus": world, "final_keys": ro.tot + CT,
            "workload": (f"cold start: {n_chunks} chunks of 704x1280 ({CT} tokens), {FORWARDS_PER_CHUNK} forwards x "
                         f"{N_LAYERS} layers each, KV budget {BUDGET} = {N_SINK} sink + {RECENT_W} recent + "
                         f"{N_LANDMARK} landmarks from a {BANK_K}-entry bank, camera returns every "
                         f"{REVISIT_EVERY} chunks; keys grow from {CT} to {LK}")}


def sp_parity(ro, dev, world, rank, group):
    """One layer through the Ulysses path (seq->head scatter with the RoPE and cache
    write, attention on this rank's heads, output rows to their owners) against
    this package's single-GPU attention over all 24 heads on the same inputs:
    every rank rebuilds the whole layer (all tokens' q/k/v, every rank's cached
    rows) and compares its token shard.  Outside the timed region."""
    import torch.distributed as dist
    from reworld_b200 import chunk_attention, rope_kv_store
    l = 0
    Ls, Hp = CT // world, HEADS // world
    start_frame = (ro.chunk * CT) // (TOK_H * TOK_W)
    rope = ro.RopeArgs(ro.table, (FRAMES, TOK_H, TOK_W), start_frame % 1000)
    tot = ro.tot

    def gather_seq(x):                 # [1, Ls, H, D] per rank -> [1, CT, H, D]
        buf = torch.empty((world * Ls, HEADS, HEAD_DIM), dtype=x.dtype, device=dev)
        dist.all_gather_into_tensor(buf, x[0].contiguous(), group=group)
        return buf.unsqueeze(0)

    def gather_heads(x):               # [1, n, Hp, D] per rank -> [1, n, H, D]
        n = x.shape[1]
        buf = torch.empty((world, n, Hp, HEAD_DIM), dtype=x.dtype, device=dev)
        dist.all_gather_into_tensor(buf, x[0].contiguous(), group=group)
        return buf.permute(1, 0, 2, 3).reshape(1, n, HEADS, HEAD_DIM)

    q_full, k_full, v_full = gather_seq(ro.q[l]), gather_seq(ro.k[l]), gather_seq(ro.v[l])
    ck = torch.zeros((1, tot + CT, HEADS, HEAD_DIM), dtype=torch.bfloat16, device=dev)
    cv = torch.zeros_like(ck)
    ck[:, :tot] = gather_heads(ro.cache_k[l][:, :tot])
    cv[:, :tot] = gather_heads(ro.cache_v[l][:, :tot])
    rope_kv_store(k_full, v_full, ck, cv, tot, rope=rope)
    ref = chunk_attention(q_full, ck, cv, rope=rope)[:, rank * Ls:(rank + 1) * Ls].float()
    y = ro.sp.layer(l, ro.q[l], ro.k[l], ro.v[l], tot, rope=rope).float()
    torch.cuda.synchronize()
    kdiff = (ro.cache_k[l][:, tot:tot + CT].float() - ck[:, tot:tot + CT, rank * Hp:(rank + 1) * Hp].float()).abs()
    err = (y - ref).abs()
    st = torch.tensor([err.max().item(), err.mean().item(), kdiff.max().item()], device=dev)
    mx = st.clone()
    dist.all_reduce(mx, op=dist.ReduceOp.MAX, group=group)
    dist.all_reduce(st, op=dist.ReduceOp.SUM, group=group)
    ok = mx[0].item() < 2e-2 and st[1].item() / world < 2e-3 and mx[2].item() == 0.0
    return {"layer": l, "keys": tot + CT, "max_abs": round(mx[0].item(), 6), "mean_abs": round(st[1].item() / world, 7),
            "cache_rows_max_abs": mx[2].item(), "tolerance": "max-abs 2e-2, mean-abs 2e-3; cache rows exact",
            "pass": bool(ok),
            "against": "reworld_b200.chunk_attention over all 24 heads on one GPU (q/k/v and cached rows of "
                       "every rank gathered), k rows roped by rw_rope_kv_store"}


def run_e2e_sp(ro, args, dev):
    """The Ulysses chunk step end to end: every rank's q/k/v sequence shard of every
    layer and forward arrives from pinned host memory, and its output shard goes
    back to pinned host memory (copies on side streams; the output is first moved
    off the shared exchange buffer on the compute stream)."""
    import torch.distributed as dist
    world = ro.world
    Ls = CT // world
    comp = torch.cuda.current_stream(dev)
    h2d = torch.cuda.Stream(dev)
    d2h = torch.cuda.Stream(dev)
    shape = (1, Ls, HEADS, HEAD_DIM)
    host_in = [torch.randn(3, *shape).to(torch.bfloat16).pin_memory() for _ in range(2)]
    host_out = [torch.empty(shape, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    dev_in = [torch.empty((3, *shape), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    dev_out = [torch.empty(shape, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_used = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    ev_read = [torch.cuda.Event() for _ in range(2)]
    for e in ev_used + ev_read:
        e.record(comp)
    bytes_in = 3 * Ls * HEADS * HEAD_DIM * 2
    bytes_out = Ls * HEADS * HEAD_DIM * 2

    def step():
        n = 0
        ro.prepare_bank()
        for _f in range(FORWARDS_PER_CHUNK):
            start_frame = (ro.chunk * CT) // (TOK_H * TOK_W)
            rope = ro.RopeArgs(ro.table, (FRAMES, TOK_H, TOK_W), start_frame % 1000)
            for l in range(N_LAYERS):
                b = n & 1
                with torch.cuda.stream(h2d):
                    h2d.wait_event(ev_used[b])
                    dev_in[b].copy_(host_in[b], non_blocking=True)
                    ev_in[b].record(h2d)
                comp.wait_event(ev_in[b])
                comp.wait_event(ev_read[b])
                y = ro.sp.layer(l, dev_in[b][0], dev_in[b][1], dev_in[b][2], ro.tot, rope=rope)
                dev_out[b].copy_(y)
                ev_used[b].record(comp)
                ev_out[b].record(comp)
                with torch.cuda.stream(d2h):
                    d2h.wait_event(ev_out[b])
                    host_out[b].copy_(dev_out[b], non_blocking=True)
                    ev_read[b].record(d2h)
                n += 1
        ro.bank_update()

    for _ in range(max(1, args.warmup // 2)):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(comp)
    for _ in range(args.steps):
        step()
    comp.wait_stream(d2h)
    t1.record(comp)
    torch.cuda.synchronize()
    t = torch.tensor([t0.elapsed_time(t1) / args.steps], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    step_flops = FORWARDS_PER_CHUNK * N_LAYERS * attn_flops(CT, LK, HEADS)
    n_io = FORWARDS_PER_CHUNK * N_LAYERS
    return {"value": round(step_flops / (ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s", "ms_per_step": round(ms, 3),
            "h2d_bytes_per_step": n_io * bytes_in * world, "d2h_bytes_per_step": n_io * bytes_out * world,
            "path": "UlyssesP2P.layer with every rank's pinned host q/k/v shard in and output shard out, copies "
                    "on side streams; bytes summed over ranks"}


def gpu_side_baselines(ro, dev):
    """Library attention on the same single-layer shape, for context: flash-attn 2
    (what the reference's attention() dispatches to on a GPU with the wheel
    installed) and torch SDPA (cuDNN on this box); plus this kernel at the
    literal 31680-key budget and the landmark gather bandwidth."""
    from reworld_b200 import chunk_attention
    out = {}
    l = 0
    q = ro.q[l]
    k = ro.cache_k[l][:, :LK].contiguous()
    v = ro.cache_v[l][:, :LK].contiguous()
    fl = attn_flops(CT, LK, HEADS)
    out["attn_ab"] = attention_ab(ro, dev)

    def timeit(fn, n=10):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(n):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / n

    ms = timeit(lambda: chunk_attention(q, k, v))
    out["attn_layer_ms"] = round(ms, 4)
    out["attn_layer_tflops"] = round(fl / ms / 1e9, 1)
    lk2 = BUDGET * CT
    ms2 = timeit(lambda: chunk_attention(q, k[:, :lk2], v[:, :lk2]))
    out["attn_layer_tflops_lk31680"] = round(attn_flops(CT, lk2, HEADS) / ms2 / 1e9, 1)
    try:
        import flash_attn
        ms3 = timeit(lambda: flash_attn.flash_attn_func(q, k, v))
        out["flash_attn2_layer_tflops"] = round(fl / ms3 / 1e9, 1)
    except Exception as ex:   # noqa: BLE001
        out["flash_attn2_layer_tflops"] = f"unavailable: {type(ex).__name__}"
    try:
        qt, kt, vt = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
        ms4 = timeit(lambda: torch.nn.functional.scaled_dot_product_attention(qt, kt, vt))
        out["torch_sdpa_layer_tflops"] = round(fl / ms4 / 1e9, 1)
    except Exception as ex:   # noqa: BLE001
        out["torch_sdpa_layer_tflops"] = f"unavailable: {type(ex).__name__}"
    # gather bandwidth: the all-layer write_into_caches of the step
    R = list(range(min(N_LANDMARK, len(ro.bank.bank))))
    msg = timeit(lambda: ro.bank.write_into_caches(ro.cache_k, ro.cache_v, R), n=5)
    nbytes = 2 * 2 * N_LAYERS * (N_SINK + RECENT_W + len(R)) * CT * ro.H * HEAD_DIM * 2   # read + write, k + v
    out["gather_ms"] = round(msg, 3)
    out["gather_gbs"] = round(nbytes / (msg * 1e-3) / 1e9, 1)
    out["rope_kv_store"] = store_measure(ro, dev, timeit)
    out["qkv_norm_rope_store"] = qkv_norm_measure(ro, dev, timeit)
    out["se3_block_apply"] = se3_measure(ro, dev, timeit)
    out["streaming_scale"] = streaming_scale(dev)
    out["host_tier"] = host_tier_measure(dev)
    # the DiT block's text cross-attention: the chunk's queries over 512 cached text keys
    kt = torch.randn(1, 512, HEADS, HEAD_DIM, device=dev).to(torch.bfloat16)
    vt = torch.randn(1, 512, HEADS, HEAD_DIM, device=dev).to(torch.bfloat16)
    msx = timeit(lambda: chunk_attention(q, kt, vt))
    out["text_cross_attn_ms"] = round(msx, 4)
    out["text_cross_attn_tflops"] = round(attn_flops(CT, 512, HEADS) / msx / 1e9, 1)
    out["block_ffn"] = ffn_measure(dev, timeit)
    out["gemm"] = gemm_ab(dev)
    out["dropin_layer"] = dropin_layer_measure(ro, dev)
    out["stress_b4"] = stress_measure(dev)
    return out


def stress_measure(dev, calls=4):
    """The stress configuration's per-layer pieces that one GPU can hold: four
    rollouts (batch 4) of 2640 queries over the 24-chunk budget split by the
    pipeline (1 sink + 7 recent + 16 landmarks = 63360 keys; 66000 with the chunk
    itself), at 24 heads and at the 3 heads one rank holds under 8-way Ulysses;
    and the bank decision (eviction + top-16 retrieval) of a full 120-entry bank.
    The whole 8-GPU rollout (a 120-entry bank of 4 rollouts is 467 GB) is not
    run here."""
    from reworld_b200 import chunk_attention
    from reworld_b200.landmark import LandmarkBankStack, budget_split
    from reworld_b200.poses import random_walk
    sp = budget_split(24, 1, 7, 120, "v15b")
    res = {"split": {"n_sink": sp.n_sink, "recent_w": sp.recent_w, "n_landmark": sp.n_landmark, "K": sp.K}}
    g = torch.Generator(device=dev).manual_seed(21)
    for lk in (sp.budget * CT, (sp.budget + 1) * CT):
        for heads in (HEADS, HEADS // 8):
            q = torch.randn(4, CT, heads, HEAD_DIM, generator=g, device=dev).to(torch.bfloat16)
            k = torch.randn(4, lk, heads, HEAD_DIM, generator=g, device=dev).to(torch.bfloat16)
            v = torch.randn(4, lk, heads, HEAD_DIM, generator=g, device=dev).to(torch.bfloat16)
            o = torch.empty_like(q)
            for _ in range(2):
                chunk_attention(q, k, v, out=o)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(calls):
                chunk_attention(q, k, v, out=o)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / calls
            res[f"attn_b4_lk{lk}_h{heads}"] = {"ms": round(ms, 4),
                                               "tflops": round(4 * attn_flops(CT, lk, heads) / ms / 1e9, 1)}
            del q, k, v, o
    # bank decisions of a 120-entry bank (tiny chunks: the decision cost does not depend on them)
    st = LandmarkBankStack.from_budget(16, 1, 1, HEAD_DIM, 24, 1, 7, 120, device=dev)
    src = torch.zeros(1, 16, 1, HEAD_DIM, dtype=torch.bfloat16, device=dev)
    cap = torch.zeros(1, 25 * 16, 1, HEAD_DIM, dtype=torch.bfloat16, device=dev)
    poses = random_walk(200, seed=8, revisit_every=8)
    times = []
    for c in range(len(poses)):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        R = st.add_chunk_from([src[0]], [src[0]], poses[c], poses[c])
        e1.record()
        torch.cuda.synchronize()
        if len(st.bank) == st.K:
            times.append(e0.elapsed_time(e1))
        st.write_into_caches([cap], [cap], R)
    res["bank120_decision_ms"] = round(statistics.median(times), 4) if times else None
    res["bank120_retrieved"] = len(R)
    res["note"] = ("batch 4 x 24 heads is the whole stress layer on one GPU; 3 heads is one rank's share at "
                   "8 GPUs; decision time = pack + rw_bank_step + host readback of one chunk, full bank")
    return res


def stress_sp_measure(dev, world, rank, group, n_layers=2, steps=3):
    """The stress configuration at N GPUs: four rollouts (batch 4) of one 2640-token
    chunk each, every one through the Ulysses layer (q/k/v scatter with k's RoPE and
    the cache write, attention of this rank's heads over the 24-chunk budget plus the
    chunk = 66000 keys, output rows to their owners), over head-sharded caches; one
    cache per (rollout, layer), n_layers layers per step.  Device time per layer of
    all four rollouts, max over ranks (a barrier on both sides of the timed steps)."""
    import torch.distributed as dist
    from reworld_b200 import RopeArgs, build_freqs, device_table
    from reworld_b200.landmark import budget_split
    from reworld_b200.ulysses import UlyssesP2P
    sp = budget_split(24, 1, 7, 120, "v15b")
    lk = (sp.budget + 1) * CT
    B = 4
    u = UlyssesP2P(group, B * n_layers, lk, CT, HEADS, HEAD_DIM, device=dev)
    g = torch.Generator(device=dev).manual_seed(900 + rank)
    for i in range(B * n_layers):
        u.caches[i].normal_(generator=g)
    Ls = CT // world
    x = [[torch.randn(1, Ls, HEADS, HEAD_DIM, generator=g, device=dev).to(torch.bfloat16) for _ in range(3)]
         for _ in range(B)]
    rope = RopeArgs(device_table(build_freqs(HEAD_DIM, 12 / 22, 20 / 40), dev), (FRAMES, TOK_H, TOK_W), 36)

    def step():
        for l in range(n_layers):
            for b in range(B):
                u.layer(b * n_layers + l, x[b][0], x[b][1], x[b][2], lk - CT, rope=rope, sync_output=False)

    step()
    step()
    u.finish()
    torch.cuda.synchronize()
    dist.barrier(group=group)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    u.finish()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / (steps * n_layers)], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    ms = float(t.item())
    dist.barrier(group=group)
    del u
    torch.cuda.synchronize()
    dist.barrier(group=group)
    return {"workload": f"stress: batch 4 rollouts x 2640 tokens, budget 24 = {sp.n_sink} sink + {sp.recent_w} recent "
                        f"+ {sp.n_landmark} landmarks (bank K {sp.K}) + the chunk = {lk} keys, 24 heads sharded "
                        f"{HEADS // world} per rank, each rollout through the Ulysses layer",
            "ms_per_layer": round(ms, 4), "tflops": round(B * attn_flops(CT, lk, HEADS) / ms / 1e9, 1),
            "n_gpus": world, "layers_timed": steps * n_layers}


def seq_kv_sp_measure(dev, world, rank, group, n_layers=3, steps=3):
    """The sequence-sharded-cache layout at N GPUs: every rank holds 31680/N of the
    cached keys for all 24 heads, and each layer moves them seq -> head with the
    chunk's q/k/v (NCCL all_to_all_single over the package's pack kernel), runs the
    attention of its 24/N heads over all 34320 keys, and sends the output back
    (ulysses.sp_chunk_attention_seq_kv).  Device time per layer (max over ranks),
    the cache exchange alone (its GB/s per GPU against NVLink's 900 GB/s per
    direction), and one layer's parity against this package's one-GPU attention
    over all heads with every rank's rows gathered."""
    import torch.distributed as dist
    from reworld_b200 import RopeArgs, build_freqs, chunk_attention, device_table, rope_kv_store
    from reworld_b200.ulysses import a2a_pack, sp_chunk_attention_seq_kv
    lc = BUDGET * CT
    Ls, Lcs, Hp = CT // world, lc // world, HEADS // world
    g = torch.Generator(device=dev).manual_seed(700 + rank)
    rnd = lambda n: torch.randn(1, n, HEADS, HEAD_DIM, generator=g, device=dev).to(torch.bfloat16)
    kv = [(rnd(Lcs), rnd(Lcs)) for _ in range(n_layers)]
    x = [(rnd(Ls), rnd(Ls), rnd(Ls)) for _ in range(n_layers)]
    work = tuple(torch.empty((1, lc + CT, Hp, HEAD_DIM), dtype=torch.bfloat16, device=dev) for _ in range(2))
    rope = RopeArgs(device_table(build_freqs(HEAD_DIM, 12 / 22, 20 / 40), dev), (FRAMES, TOK_H, TOK_W), BUDGET * FRAMES)

    def step():
        for l in range(n_layers):
            sp_chunk_attention_seq_kv(x[l][0], x[l][1], x[l][2], kv[l][0], kv[l][1], rope=rope, group=group,
                                      work=work)

    def exchange():
        for l in range(n_layers):
            for t, dst in zip(kv[l], work):
                dist.all_to_all_single(dst[:, :lc].view(world, 1, Lcs, Hp, HEAD_DIM), a2a_pack(t, world),
                                       group=group)

    def timed(fn):
        fn()
        torch.cuda.synchronize()
        dist.barrier(group=group)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / (steps * n_layers)], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        return float(t.item())

    step()
    ms = timed(step)
    ms_x = timed(exchange)
    # parity: layer 0 against one GPU's attention over all heads (outside the timed region)
    def gather_seq(t):
        buf = torch.empty((world * t.shape[1], HEADS, HEAD_DIM), dtype=t.dtype, device=dev)
        dist.all_gather_into_tensor(buf, t[0].contiguous(), group=group)
        return buf.unsqueeze(0)
    q_f, k_f, v_f = (gather_seq(t) for t in x[0])
    ck = torch.empty((1, lc + CT, HEADS, HEAD_DIM), dtype=torch.bfloat16, device=dev)
    cv = torch.empty_like(ck)
    ck[:, :lc], cv[:, :lc] = gather_seq(kv[0][0]), gather_seq(kv[0][1])
    rope_kv_store(k_f, v_f, ck, cv, lc, rope=rope)
    ref = chunk_attention(q_f, ck, cv, rope=rope)[:, rank * Ls:(rank + 1) * Ls].float()
    y = sp_chunk_attention_seq_kv(x[0][0], x[0][1], x[0][2], kv[0][0], kv[0][1], rope=rope, group=group,
                                  work=work).float()
    err = (y - ref).abs()
    st = torch.tensor([err.max().item(), err.mean().item()], device=dev)
    mx = st.clone()
    dist.all_reduce(mx, op=dist.ReduceOp.MAX, group=group)
    dist.all_reduce(st, op=dist.ReduceOp.SUM, group=group)
    del ck, cv, ref, kv, work
    torch.cuda.synchronize()
    dist.barrier(group=group)
    x_bytes = 2 * Lcs * HEADS * HEAD_DIM * 2 * (world - 1) // world      # cache K + V sent per GPU per layer
    qkvo_bytes = 4 * Ls * HEADS * HEAD_DIM * 2 * (world - 1) // world     # q, k, v in and the output back
    return {"workload": f"cache sharded along the sequence: {lc} cached keys / {world} ranks, all 24 heads each; "
                        f"per layer the cache and the chunk's q/k/v go seq -> head (NCCL all_to_all_single), "
                        f"attention of {Hp} heads over {lc + CT} keys, output back",
            "ms_per_layer": round(ms, 4), "tflops": round(attn_flops(CT, lc + CT, HEADS) / ms / 1e9, 1),
            "cache_exchange_ms_per_layer": round(ms_x, 4),
            "cache_exchange_bytes_per_gpu": x_bytes, "qkvo_exchange_bytes_per_gpu": qkvo_bytes,
            "cache_exchange_gbs_per_gpu": round(x_bytes / (ms_x * 1e-3) / 1e9, 1),
            "nvlink_peak_gbs_per_direction": 900.0,
            "parity": {"max_abs": round(mx[0].item(), 6), "mean_abs": round(st[1].item() / world, 7),
                       "pass": bool(mx[0].item() < 2e-2 and st[1].item() / world < 2e-3),
                       "tolerance": "max-abs 2e-2, mean-abs 2e-3",
                       "against": "reworld_b200.chunk_attention over all 24 heads on one GPU, every rank's rows gathered"},
            "n_gpus": world, "layers_timed": steps * n_layers}


def gemm_ab(dev, reps=9, calls=8, n_inputs=3):
    """rw_gemm_bf16 against cuBLAS (torch.nn.functional.linear) on the projections of
    one layer-chunk (2640 tokens, width 3072): the stacked q|k|v GEMM, value_proj,
    the stacked o|prope_proj GEMM over [y | P y], and the FFN pair (the first with the
    tanh GELU: in the epilogue here, a separate torch op after cuBLAS).  Interleaved
    rounds on inputs rotating over n_inputs copies; median round per arm."""
    from reworld_b200.gemm import linear
    C = HEADS * HEAD_DIM
    shapes = [("qkv", CT, 3 * C, C, False), ("value_proj", CT, C, C, False), ("o_prope", CT, C, 2 * C, False),
              ("ffn_up_gelu", CT, 14336, C, True), ("ffn_down", CT, C, 14336, False)]
    burst = load_peaks()[0]
    res = {}
    g = torch.Generator(device=dev).manual_seed(9)
    for name, M, N, K, gelu in shapes:
        xs = [torch.randn(M, K, generator=g, device=dev).to(torch.bfloat16) for _ in range(n_inputs)]
        ws = [(torch.randn(N, K, generator=g, device=dev) * 0.02).to(torch.bfloat16) for _ in range(n_inputs)]
        bs = [(torch.randn(N, generator=g, device=dev) * 0.02).to(torch.bfloat16) for _ in range(n_inputs)]
        outs = [torch.empty(M, N, dtype=torch.bfloat16, device=dev) for _ in range(n_inputs)]

        def ours(i, gelu=gelu):
            linear(xs[i], ws[i], bs[i], gelu=gelu, out=outs[i])

        def cublas(i, gelu=gelu):
            y = torch.nn.functional.linear(xs[i], ws[i], bs[i])
            if gelu:
                torch.nn.functional.gelu(y, approximate="tanh")

        arms = {"reworld_b200": ours, "cublas": cublas}
        for f in arms.values():
            for i in range(n_inputs):
                f(i)
        torch.cuda.synchronize()
        times = {a: [] for a in arms}
        for _ in range(reps):
            for a, f in arms.items():
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for c in range(calls):
                    f(c % n_inputs)
                e1.record()
                e1.synchronize()
                times[a].append(e0.elapsed_time(e1) / calls)
        fl = 2.0 * M * N * K
        r = {"shape": f"[{M}, {K}] x [{N}, {K}]^T" + (" + GELU(tanh)" if gelu else "")}
        for a, ts in times.items():
            med = statistics.median(ts)
            r[a] = {"us": round(med * 1e3, 1), "tflops": round(fl / med / 1e9, 1)}
        r["ratio_vs_cublas"] = round(statistics.median(times["cublas"]) / statistics.median(times["reworld_b200"]), 3)
        r["frac_of_bf16_burst"] = round(fl / statistics.median(times["reworld_b200"]) / 1e9 / burst, 4)
        res[name] = r
    res["method"] = f"{reps} interleaved rounds of {calls} calls per arm, median; inputs rotate over {n_inputs} copies"
    return res


def dropin_layer_measure(ro, dev, n_calls=6):
    """One layer of the installed self-attention drop-in (prop_self_attn_forward at
    the 5B width: 3072 channels, 24 heads, a 2640-token chunk over a 12-chunk cache,
    with a camera context so the PRoPE path runs) called the way the reference model
    calls it, with its input x copied from pinned host memory and its output copied
    back to pinned host memory inside the timed region: the plugin's own overheads
    (index bookkeeping, launches, host work) included.  Per call, against the
    attention kernel alone on the same shape."""
    import torch.nn as nn
    from reworld_b200.self_attn import install, write_index
    from reworld_b200.poses import random_walk
    C = HEADS * HEAD_DIM

    class _RMS(nn.Module):
        def __init__(self):
            super().__init__()
            self.eps = 1e-6
            self.weight = nn.Parameter(torch.ones(C))

    class _Attn(nn.Module):
        def __init__(self):
            super().__init__()
            self.num_heads, self.head_dim = HEADS, HEAD_DIM
            self.local_attn_size, self.sink_size, self.max_attention_size = -1, 0, None
            self.q, self.k, self.v, self.o = (nn.Linear(C, C) for _ in range(4))
            self.norm_q, self.norm_k = _RMS(), _RMS()
            self.pose_mlp = nn.Sequential(nn.Linear(12, 256), nn.SiLU(), nn.Linear(256, HEAD_DIM // 2))
            self.value_proj, self.prope_proj = nn.Linear(C, C), nn.Linear(C, C)

    g = torch.Generator().manual_seed(4)
    mod = _Attn()
    with torch.no_grad():
        for p_ in mod.parameters():
            p_.copy_(torch.randn(p_.shape, generator=g) * 0.02)
    mod = mod.to(device=dev, dtype=torch.bfloat16)
    install([type("Blk", (), {"self_attn": mod})()])
    n0 = LK - CT
    cache = {"k": ro.cache_k[0], "v": ro.cache_v[0], "global_end_index": torch.tensor([n0], device=dev),
             "local_end_index": torch.tensor([n0], device=dev)}
    frames = random_walk(n0 // (TOK_H * TOK_W) + FRAMES, seed=3)
    ctx = torch.from_numpy(np.stack(frames)).unsqueeze(0).to(device=dev, dtype=torch.bfloat16)
    freqs = __import__("reworld_b200").build_freqs(HEAD_DIM, 12 / 22, 20 / 40)
    x_host = torch.randn(1, CT, C).to(torch.bfloat16).pin_memory()
    y_host = torch.empty(1, CT, C, dtype=torch.bfloat16).pin_memory()
    seq_lens, grid = torch.tensor([CT]), torch.tensor([[FRAMES, TOK_H, TOK_W]])

    x_dev = x_host.to(dev)

    def call(host_io):
        # the same chunk position every call (written the way the forward writes the
        # indices, so their host mirrors stay valid and no call reads them back)
        write_index(cache["global_end_index"], n0)
        write_index(cache["local_end_index"], n0)
        x = x_host.to(dev, non_blocking=True) if host_io else x_dev
        y = mod.forward(x, seq_lens, grid, freqs, None, kv_cache=cache, current_start=n0, prope_context=ctx)
        if host_io:
            y_host.copy_(y, non_blocking=True)

    res = {}
    with torch.no_grad():
        for host_io in (False, True):
            for _ in range(2):
                call(host_io)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(n_calls):
                call(host_io)
            e1.record()
            torch.cuda.synchronize()
            res[host_io] = (e0.elapsed_time(e1) / n_calls, (time.perf_counter() - t0) / n_calls)
    ms, wall = res[False]
    ms_io, _ = res[True]
    fl_attn = attn_flops(CT, LK, HEADS)
    fl_proj = 2.0 * CT * C * (3 * C + C + 2 * C)           # q|k|v, value_proj, o|prope_proj
    return {"ms_per_layer": round(ms, 4), "host_wall_ms_per_layer": round(wall * 1e3, 4),
            "tflops": round((fl_attn + fl_proj) / (ms * 1e-3) / 1e12, 1),
            "e2e_ms_per_layer": round(ms_io, 4), "h2d_bytes": CT * C * 2, "d2h_bytes": CT * C * 2,
            "path": "installed prop_self_attn_forward (stacked q|k|v GEMM, fused RMSNorm/RoPE/cache store, PRoPE "
                    "SE3 + value_proj GEMM with residual, attention writing y and P y, [y | P y] GEMM) as the model "
                    "calls it, x on the "
                    "device; e2e_ms_per_layer: x from pinned host memory and the output back to it on the same stream",
            "shape": f"x [1, {CT}, {C}], cache {LK} keys x {HEADS} heads, PRoPE context on"}


def attention_ab(ro, dev, reps=7, calls=6, n_inputs=3):
    """This package's chunk attention against the library attention the reference
    would run on this GPU (torch SDPA: cuDNN here; flash-attn 2, the wheel the
    reference's attention() dispatches to), A/B interleaved: `reps` rounds, each
    timing `calls` back-to-back calls of every arm in turn on the same inputs,
    which rotate over n_inputs layers' q and contiguous K/V (422 MB each, so
    every call reads from HBM).  Reports each arm's median round."""
    from reworld_b200 import chunk_attention
    fl = attn_flops(CT, LK, HEADS)
    sets = []
    for i in range(n_inputs):
        l = i % N_LAYERS
        sets.append((ro.q[l], ro.cache_k[l][:, :LK].contiguous(), ro.cache_v[l][:, :LK].contiguous()))
    sdpa_sets = [(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)) for q, k, v in sets]
    outs = [torch.empty_like(q) for q, _, _ in sets]
    arms = {"reworld_b200": lambda i: chunk_attention(*sets[i], out=outs[i]),
            "torch_sdpa": lambda i: torch.nn.functional.scaled_dot_product_attention(*sdpa_sets[i])}
    try:
        import flash_attn
        arms["flash_attn2"] = lambda i: flash_attn.flash_attn_func(*sets[i])
    except Exception:   # noqa: BLE001 - the wheel is optional
        pass
    for fn in arms.values():                      # warm-up (library autotuning, workspace growth)
        for i in range(n_inputs):
            fn(i)
    torch.cuda.synchronize()
    times = {name: [] for name in arms}
    for _ in range(reps):
        for name, fn in arms.items():
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for c in range(calls):
                fn(c % n_inputs)
            b.record()
            b.synchronize()
            times[name].append(a.elapsed_time(b) / calls)
    res = {}
    for name, ts in times.items():
        med = statistics.median(ts)
        res[name] = {"median_ms": round(med, 4), "tflops": round(fl / med / 1e9, 1),
                     "rounds_ms": [round(t, 4) for t in ts]}
    res["speedup_vs_torch_sdpa"] = round(res["torch_sdpa"]["median_ms"] / res["reworld_b200"]["median_ms"], 3)
    res["shape"] = f"q [1, {CT}, {HEADS}, {HEAD_DIM}], k/v [1, {LK}, {HEADS}, {HEAD_DIM}] bf16"
    res["method"] = (f"{reps} interleaved rounds of {calls} calls per arm, inputs rotating over {n_inputs} "
                     f"layers (each > L2); median round")
    return res


def ffn_measure(dev, timeit, ffn_dim=14336):
    """The DiT block's norm2 + FFN on one layer's chunk [2640, 3072]: the LayerNorm row
    kernel, and GeluFFN (two rw_gemm_bf16 GEMMs, the GELU in the first one's
    epilogue) against the reference's Linear -> GELU(tanh) -> Linear (cuBLAS and a
    torch GELU), both on the same bf16 weights."""
    import torch.nn as nn
    from reworld_b200.block import GeluFFN, row_norm
    C = HEADS * HEAD_DIM
    seq = nn.Sequential(nn.Linear(C, ffn_dim), nn.GELU(approximate="tanh"), nn.Linear(ffn_dim, C))
    seq = seq.to(device=dev, dtype=torch.bfloat16)
    fused = GeluFFN(seq)
    xs = [torch.randn(1, CT, C, device=dev).to(torch.bfloat16) for _ in range(8)]
    it = [0]

    def nxt():
        it[0] += 1
        return xs[it[0] % len(xs)]

    outs = [torch.empty_like(x) for x in xs]
    with torch.no_grad():
        ms_f = timeit(lambda: fused(nxt()), n=10)
        ms_u = timeit(lambda: seq(nxt()), n=10)
        # a launch of a few microseconds: timed from CUDA-graph replays, not a Python loop
        g_n = _graph(dev, lambda i: row_norm(xs[i], None, None, 1e-6, "layer", out=outs[i]), len(xs))
        ms_n = timeit(g_n.replay, n=8) / len(xs)
    fl = 2 * 2 * CT * C * ffn_dim
    burst, sustained, hbm, peak_src = load_peaks()
    nb = 2 * CT * C * 2
    return {"ffn_ms": round(ms_f, 4), "ffn_tflops": round(fl / ms_f / 1e9, 1),
            "frac_of_bf16_burst": round(fl / ms_f / 1e9 / burst, 4), "reference_ffn_ms": round(ms_u, 4),
            "layer_norm_ms": round(ms_n, 4), "layer_norm_gbs": round(nb / (ms_n * 1e-3) / 1e9, 1),
            "shape": f"[{CT}, {C}] -> {ffn_dim} -> {C}, bf16; inputs rotate over 8 chunks",
            "peak_kind": f"cuBLAS bf16 burst ({peak_src})", "reference_ffn": "nn.Sequential on cuBLAS + torch GELU"}


def host_tier_measure(dev, n_layers=2, chunks=20):
    """The bank with pinned-host master copies (the reference's default direct
    mode, and the staged hot set) at the chunk shape, on a 2-layer stack to bound
    the pinned host pool: per chunk step (pack, decision, write-through, prefetch,
    assembly of sink | recent | bank[R] into each layer's cache) timed on the
    compute stream after the bank is full, and the host-to-device bytes it moved."""
    from reworld_b200.landmark import LandmarkBankStack
    from reworld_b200.poses import random_walk
    res = {}
    poses = random_walk(chunks + 2, seed=5, revisit_every=4)
    for mode, hot in (("direct", 0), ("staged", N_LANDMARK)):
        st = LandmarkBankStack(CT, n_layers, HEADS, HEAD_DIM, n_sink=N_SINK, recent_w=RECENT_W, K=8,
                               retrieve_k=N_LANDMARK, device=dev, host_tier=True, hot_gpu=hot)
        src = [torch.randn(2, CT, HEADS, HEAD_DIM, device=dev).to(torch.bfloat16) for _ in range(n_layers)]
        caps = [torch.zeros(1, (BUDGET + 1) * CT, HEADS, HEAD_DIM, dtype=torch.bfloat16, device=dev)
                for _ in range(2 * n_layers)]
        times, h2d = [], []
        for c in range(chunks):
            b0 = st.tier.counters["bytes_h2d"]
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            R = st.add_chunk_from([x[0] for x in src], [x[1] for x in src], poses[c], poses[c + 1])
            st.write_into_caches(caps[:n_layers], caps[n_layers:], R)
            e1.record()
            torch.cuda.synchronize()
            if c >= N_SINK + RECENT_W + 8:          # bank full: steady state
                times.append(e0.elapsed_time(e1))
                h2d.append(st.tier.counters["bytes_h2d"] - b0)
        ms = statistics.median(times)
        res[mode] = {"ms_per_chunk": round(ms, 3), "h2d_bytes_per_chunk": int(statistics.median(h2d)),
                     "h2d_gbs": round(statistics.median(h2d) / (ms * 1e-3) / 1e9, 1), "hot_gpu": hot}
        del st
    res["config"] = (f"{n_layers} layers x [{CT}, {HEADS}, {HEAD_DIM}] bf16 K and V per chunk, bank K = 8, "
                     f"retrieve {N_LANDMARK}, sink {N_SINK}, recent {RECENT_W}; median of the steady-state chunks")
    return res


def _graph(dev, fn, n):
    """fn() called n times, captured once (after one uncaptured round on a side stream)."""
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for i in range(n):
            fn(i)
    torch.cuda.current_stream(dev).wait_stream(side)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        for i in range(n):
            fn(i)
    return gr


def store_measure(ro, dev, timeit, n_rot=8):
    """rw_rope_kv_store as the chunk step runs it (RoPE of k, cache write of k and v
    for one layer's chunk), launches rotating over n_rot layers' k/v and caches
    (more than L2), timed from CUDA-graph replays."""
    from reworld_b200 import rope_kv_store
    rope = ro.RopeArgs(ro.table, (FRAMES, TOK_H, TOK_W), 0)
    g = _graph(dev, lambda i: rope_kv_store(ro.k[i], ro.v[i], ro.cache_k[i], ro.cache_v[i], ro.tot, rope=rope),
               n_rot)
    ms = timeit(g.replay, n=8) / n_rot
    nbytes = 4 * CT * HEADS * HEAD_DIM * 2          # k and v read, both cache rows written
    _, _, hbm, peak_src = load_peaks()
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"ms": round(ms, 4), "gbs": round(gbs, 1), "bytes_per_launch": nbytes, "frac_of_hbm": round(gbs / hbm, 4),
            "peak_kind": f"copy bandwidth ({peak_src})", "timing": "CUDA graph replay, per launch"}


def se3_measure(ro, dev, timeit, n_rot=8):
    """The PRoPE SE3 transform of one layer's chunk activations [1, 2640, 24, 128]
    (rw_se3_block_apply) against the reference's torch formulation of
    _se3_block_apply on the same inputs; launches rotate over n_rot layers'
    activations (n_rot x 16.2 MB, more than L2), timed from CUDA-graph replays."""
    from reworld_b200 import _native
    from reworld_b200._native import c_vp
    from reworld_b200.self_attn import _se3_torch, se3_block_apply, se3_mats
    ctx = torch.eye(4, device=dev).repeat(1, 5, 1, 1)
    ctx[..., :3, 3] = torch.tensor([0.3, -0.2, 1.1], device=dev)
    outs = [torch.empty_like(ro.q[i]) for i in range(n_rot)]
    mats = se3_mats(ctx, "P", FRAMES, torch.bfloat16)
    lib = _native.lib()

    def kernel(i):
        x, o = ro.q[i], outs[i]
        _native.check(lib.rw_se3_block_apply(c_vp(x.data_ptr()), c_vp(o.data_ptr()), c_vp(mats.data_ptr()), 1, CT,
                                             HEADS, HEAD_DIM, TOK_H * TOK_W, *x.stride()[:3], *o.stride()[:3],
                                             _native.stream_ptr(dev)), "rw_se3_block_apply")

    g_k = _graph(dev, kernel, n_rot)
    g_p = _graph(dev, lambda i: se3_block_apply(ro.q[i], ctx, "P", TOK_H * TOK_W, out=outs[i]), n_rot)
    g_t = _graph(dev, lambda i: _se3_torch(ro.q[i], ctx, "P", TOK_H * TOK_W), n_rot)
    ms_k = timeit(g_k.replay, n=8) / n_rot
    ms_p = timeit(g_p.replay, n=8) / n_rot
    ms_t = timeit(g_t.replay, n=8) / n_rot
    nbytes = 2 * CT * HEADS * HEAD_DIM * 2
    _, _, hbm, peak_src = load_peaks()
    gbs = nbytes / (ms_k * 1e-3) / 1e9
    return {"ms": round(ms_k, 4), "gbs": round(gbs, 1), "bytes_per_launch": nbytes,
            "frac_of_hbm": round(gbs / hbm, 4), "peak_kind": f"copy bandwidth ({peak_src})",
            "public_call_ms": round(ms_p, 4), "torch_ms": round(ms_t, 4), "speedup_vs_torch": round(ms_t / ms_p, 2),
            "shape": f"1 x {CT} tokens x 24 heads x 128, 3 frames",
            "timing": "CUDA graph replay, per launch; ms = the kernel, public_call_ms adds the frame matrices' "
                      "preparation (a few small torch kernels per call)"}


def _torch_rms(x, w, eps=1e-6):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)).type_as(x) * w


def qkv_norm_measure(ro, dev, timeit, n_rot=4):
    """The step before the attention for one layer's chunk (2640 tokens x 3072):
    q/k RMSNorm + RoPE of k + cache write of k and v, as one rw_qkv_norm_rope_store
    launch, against the unfused path it replaces on the same inputs (torch's two
    WanRMSNorm evaluations + rw_rope_kv_store).  The launches rotate over n_rot
    layers' inputs and caches (n_rot x 48.7 MB of q|k|v rows, more than L2)."""
    from reworld_b200 import qkv_norm_rope_store, rope_kv_store
    C = HEADS * HEAD_DIM
    g = torch.Generator(device=dev).manual_seed(77)
    qkv = [(torch.randn(1, CT, 3 * C, generator=g, device=dev) * 1.5).to(torch.bfloat16) for _ in range(n_rot)]
    wq = (1 + 0.05 * torch.randn(C, generator=g, device=dev)).to(torch.bfloat16)
    wk = (1 + 0.05 * torch.randn(C, generator=g, device=dev)).to(torch.bfloat16)
    qo = [torch.empty(1, CT, HEADS, HEAD_DIM, dtype=torch.bfloat16, device=dev) for _ in range(n_rot)]
    rope = ro.RopeArgs(ro.table, (FRAMES, TOK_H, TOK_W), 0)
    it = [0]

    def fused():
        i = it[0] % n_rot
        it[0] += 1
        x = qkv[i]
        qkv_norm_rope_store(x[..., :C], x[..., C:2 * C], x[..., 2 * C:], wq, wk, ro.cache_k[i], ro.cache_v[i],
                            ro.tot, 1e-6, rope=rope, q_out=qo[i])

    def unfused():
        i = it[0] % n_rot
        it[0] += 1
        x = qkv[i]
        _torch_rms(x[..., :C], wq)
        k = _torch_rms(x[..., C:2 * C], wk).view(1, CT, HEADS, HEAD_DIM)
        rope_kv_store(k, x[..., 2 * C:].view(1, CT, HEADS, HEAD_DIM), ro.cache_k[i], ro.cache_v[i], ro.tot,
                      rope=rope)

    def graph_of(fn):
        # the n_rot calls captured once: replays time the GPU work, not the Python around it
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(n_rot):
                fn()
        torch.cuda.current_stream(dev).wait_stream(side)
        it[0] = 0
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            for _ in range(n_rot):
                fn()
        return gr

    g_f, g_u = graph_of(fused), graph_of(unfused)
    ms_f = timeit(g_f.replay, n=8) / n_rot
    ms_u = timeit(g_u.replay, n=8) / n_rot
    nbytes = CT * C * 2 * 6 + 2 * C * 2          # q, k, v rows in; q, k, v rows out; two weight vectors
    _, _, hbm, peak_src = load_peaks()
    gbs = nbytes / (ms_f * 1e-3) / 1e9
    return {"ms": round(ms_f, 4), "gbs": round(gbs, 1), "bytes_per_launch": nbytes,
            "frac_of_hbm": round(gbs / hbm, 4), "hbm_peak_gbs": hbm, "peak_kind": f"copy bandwidth ({peak_src})",
            "unfused_ms": round(ms_u, 4), "speedup_vs_unfused": round(ms_u / ms_f, 2),
            "shape": f"1 x {CT} tokens x {C} (24 heads x 128), RoPE on k, cache write at row {ro.tot}",
            "unfused": "torch WanRMSNorm formula on q and k (GPU) + rw_rope_kv_store",
            "timing": f"CUDA graph of {n_rot} launches over {n_rot} layers' inputs and caches, replayed; "
                      "per launch"}


def streaming_scale(dev, batches=(1, 2, 4, 8)):
    """The two streaming kernels of a layer-chunk over 1..8 chunks at once (batch
    B): time = a fixed part per launch + a part per chunk; the per-chunk slope's
    bandwidth is what the inner loop streams at.  CUDA-graph replay, inputs
    rotating over two copies (each > L2 from B = 2 on)."""
    from reworld_b200 import RopeArgs, build_freqs, device_table, qkv_norm_rope_store, rope_kv_store
    C = HEADS * HEAD_DIM
    g = torch.Generator(device=dev).manual_seed(5)
    rope = RopeArgs(device_table(build_freqs(HEAD_DIM, 12 / 22, 20 / 40), dev), (FRAMES, TOK_H, TOK_W), 36)
    wq = (1 + 0.05 * torch.randn(C, generator=g, device=dev)).to(torch.bfloat16)
    res = {"norm_us": [], "store_us": []}
    for B in batches:
        x = [(torch.randn(B, CT, 3 * C, generator=g, device=dev) * 1.5).to(torch.bfloat16) for _ in range(2)]
        ck = [torch.zeros(B, 2 * CT, HEADS, HEAD_DIM, dtype=torch.bfloat16, device=dev) for _ in range(2)]
        cv = [torch.zeros_like(c) for c in ck]
        qo = [torch.empty(B, CT, HEADS, HEAD_DIM, dtype=torch.bfloat16, device=dev) for _ in range(2)]
        fns = {"norm_us": lambda i: qkv_norm_rope_store(x[i][..., :C], x[i][..., C:2 * C], x[i][..., 2 * C:], wq, wq,
                                                         ck[i], cv[i], CT, 1e-6, rope=rope, q_out=qo[i]),
               "store_us": lambda i: rope_kv_store(x[i][..., C:2 * C].view(B, CT, HEADS, HEAD_DIM),
                                                   x[i][..., 2 * C:].view(B, CT, HEADS, HEAD_DIM), ck[i], cv[i], CT,
                                                   rope=rope)}
        for key, fn in fns.items():
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                fn(0)
                fn(1)
            torch.cuda.current_stream(dev).wait_stream(side)
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                fn(0)
                fn(1)
            ts = []
            for _ in range(5):
                for _ in range(2):
                    gr.replay()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda.synchronize()
                a.record()
                for _ in range(10):
                    gr.replay()
                b.record()
                torch.cuda.synchronize()
                ts.append(a.elapsed_time(b) / 20)
            res[key].append(round(1e3 * sorted(ts)[2], 2))
        del x, ck, cv, qo
    _, _, hbm, _ = load_peaks()
    for key, nb in (("norm", CT * C * 12), ("store", CT * C * 8)):
        t = res[f"{key}_us"]
        slope = (t[-1] - t[0]) / (batches[-1] - batches[0])
        res[f"{key}_slope_gbs"] = round(nb / (slope * 1e-6) / 1e9, 1)
        res[f"{key}_slope_frac_of_hbm"] = round(nb / (slope * 1e-6) / 1e9 / hbm, 3)
        res[f"{key}_fixed_us"] = round(t[0] - slope, 2)
    res["batches"] = list(batches)
    res["bytes_per_chunk"] = {"norm": CT * C * 12, "store": CT * C * 8}
    return res


# ------------------------------------------------------------------ CPU baseline / reference arm
def cpu_sample(heads, lq=CT, lk=LK, seed=0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(1, lq, heads, HEAD_DIM, generator=g).to(torch.bfloat16)
    k = torch.randn(1, lk, heads, HEAD_DIM, generator=g).to(torch.bfloat16)
    v = torch.randn(1, lk, heads, HEAD_DIM, generator=g).to(torch.bfloat16)
    return q, k, v


def cpu_baseline(budget_s=15.0):
    """The reference's CPU attention path (oracle port of wan_5b/modules/attention.py:
    164-179, torch SDPA in bf16) on this host's cores, on a bounded sample of
    the workload: whole layers (24 heads, Lq 2640 x Lk 34320) repeated for about
    budget_s seconds."""
    from oracle.attention import reference_attention_cpu
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    q, k, v = cpu_sample(HEADS)
    t = time.perf_counter()
    reference_attention_cpu(q, k, v)                 # warm-up, also sizes the sample
    one = time.perf_counter() - t
    reps = max(1, int(budget_s / max(one, 1e-3)))
    t = time.perf_counter()
    for _ in range(reps):
        reference_attention_cpu(q, k, v)
    dt = (time.perf_counter() - t) / reps
    fl = attn_flops(CT, LK, HEADS)
    return {"value": round(fl / dt / 1e12, 4), "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": f"{reps} layers (24 heads, Lq {CT} x Lk {LK}) of bf16 torch SDPA on CPU after 1 warm-up, "
                      f"{dt:.3f} s per layer ({reps * dt:.1f} s total)"}


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle.attention import reference_attention_cpu
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    q, k, v = cpu_sample(HEADS)
    t = time.perf_counter()
    reference_attention_cpu(q, k, v)
    one = time.perf_counter() - t
    # each step: whole layers of the chunk, as many as fit in the CPU budget spread over the run
    per_step = max(one, args.cpu_seconds / max(1, args.steps + args.warmup))
    layers = max(1, min(N_LAYERS * FORWARDS_PER_CHUNK, int(per_step / max(one, 1e-3))))
    for _ in range(args.warmup):
        for _l in range(layers):
            reference_attention_cpu(q, k, v)
    t = time.perf_counter()
    for _ in range(args.steps):
        for _l in range(layers):
            reference_attention_cpu(q, k, v)
    dt = (time.perf_counter() - t) / args.steps
    fl = layers * attn_flops(CT, LK, HEADS)
    val = round(fl / dt / 1e12, 4)
    sample = (f"{layers} layers (24 heads, Lq {CT} x Lk {LK}) per step of bf16 torch SDPA on CPU "
              f"(the reference attention() branch without flash-attention), {dt:.2f} s per step")
    line = {"impl": "reference", "metric": METRIC, "value": val, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3),
            "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded N(0,1))",
            "config": {"workload": WORKLOAD, "Lq": CT, "Lk": LK, "layers": N_LAYERS, "heads": HEADS,
                       "head_dim": HEAD_DIM, "parallelism": "cpu"},
            "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
