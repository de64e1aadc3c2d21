"""Benchmark of the paged INT8 KV-cache hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1)

Prints one JSON line on rank 0.  The headline is the fused paged verify
attention at the Llama-3.1-8B shape (32 query / 8 KV heads, head_dim 128,
window 5, 32 sequences per GPU with contexts uniform in [1024, 8192], block
size 16, randomly permuted physical blocks): HBM GB/s of algorithmic bytes
(INT8 K/V codes + fp32 scales of every cached token, query, output and table
entries) over the device time of the attention launches, summed over ranks
(requests are data-parallel: every rank serves its own 32 sequences, no
collective).  The same line carries the append workload (32 layers, 256
sequences appending a 5-token window per step, 0-5 tokens rolled back each,
65536-block pool with a randomized free list) as tokens/s.

Inputs are synthetic (seeded N(0,1) K/V and queries, there is no dataset for
this path).  L2 is flushed (a 256 MiB write) between timed iterations, and
each pool is larger than L2.  ``--impl reference`` times the reference's own
CPU path on this host (its unchanged Python package and C++ quantizer,
copied and built into oracle/_ref by ``make -C oracle ref``): its
submit_paged_attention on CPU torch with all host threads (the headline
value), its materialize_legacy_cache reconstruct path with torch CPU SDPA,
and its PagedKVCache append / truncate with NativeKVQuantizer, each on a
bounded sample of the same workloads.  The same measurements are reported
beside this library's numbers as ``cpu_baseline`` blocks.
"""

from __future__ import annotations

import argparse
import gc
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "llm-inference-accelerator_b200"))

METRIC = "paged INT8 verify-attn HBM GB/s (% of peak) at 1/2/4/8 B200; append tokens/s"
VERIFY = dict(batch=32, query_heads=32, kv_heads=8, head_dim=128, window=5, block_size=16,
              min_context=1024, max_context=8192)
APPEND = dict(layers=32, kv_heads=8, head_dim=128, sequences=256, window=5, block_size=16, num_blocks=65536)
LONG = dict(batch=8, query_heads=64, kv_heads=8, head_dim=128, window=5, block_size=16, context=131072)
# end-to-end speculative decoding: random-init Llama-architecture draft and
# target (bf16, weights N(0, 0.02)), uniform random prompt ids
SPEC = dict(batch=64, prompt=1024, new_tokens=64, window=5, min_window=4, max_window=8, temperature=1.0,
            vocab=128256,
            draft=dict(layers=16, hidden=2048, heads=32, kv_heads=8, head_dim=64, intermediate=8192),
            target=dict(layers=32, hidden=4096, heads=32, kv_heads=8, head_dim=128, intermediate=14336))
# the CPU-runnable workload of the reference: 4 sequences prefill 512 fp32
# tokens, then 64 rounds append a 5-token window each and keep the prefix
# accepted by Bernoulli(0.7) draws up to the first rejection
CONFIG1 = dict(layers=16, kv_heads=8, head_dim=64, block_size=16, num_blocks=4096, sequences=4, prefill=512,
               rounds=64, window=5, accept_p=0.7)
VERIFY_WORKLOAD = ("8B verify attention: B32 Hq32 Hkv8 D128 window5 ctx U[1024,8192] bs16, "
                   "randomly permuted physical blocks, one layer")
FLUSH_BYTES = 256 << 20
HOLD_CYCLES = 200_000  # about 0.1 ms of device time at B200 clocks


def hold_device():
    """Occupy the stream for ~0.1 ms before a start event is recorded, so the
    host has queued the timed launches (Python and ctypes call overhead)
    before the start event executes: the events then bracket device work
    only, never a gap where the device waits for the host."""
    import torch

    torch.cuda._sleep(HOLD_CYCLES)


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--seed", type=int, default=2024)
    p.add_argument("--skip-append", action="store_true", help="measure only the verify attention")
    p.add_argument("--skip-cpu-baseline", action="store_true")
    p.add_argument("--skip-config1", action="store_true",
                   help="skip the CPU-runnable workload (16 layers, 4 sequences, 64 speculative rounds) on the GPU")
    p.add_argument("--skip-long", action="store_true", help="skip the 70B long-context (KV-head parallel) workload")
    p.add_argument("--skip-speculative", action="store_true",
                   help="skip the end-to-end speculative decoding workload (draft 16L d2048 / target 32L d4096)")
    p.add_argument("--profile-append", action="store_true",
                   help="the append workload's step (256 sequences x 5 tokens, 32 layers) on a 4096-block pool, "
                        "a few steps, no timing: small enough for a full ncu capture")
    p.add_argument("--skip-device-pages", action="store_true",
                   help="skip the append workload's step through the device-resident page allocator")
    p.add_argument("--skip-sampling", action="store_true",
                   help="skip the device acceptance/sampling workload (64 sequences x 6 proposals x 128256 tokens)")
    p.add_argument("--profile-sampling", action="store_true",
                   help="the acceptance/sampling workload only, a few rounds, no timing: for ncu")
    p.add_argument("--profile-case", choices=("decode", "gather", "simt", "pages"),
                   help="a few untimed calls of one kernel family for ncu: decode-shape attention (64 sequences "
                        "x ~1100 tokens, head_dim 128 and 64, windows 1 and 6), the gather-dequantize of the "
                        "verify batch, the CUDA-core attention kernel (head_dim 256), or the device allocator's "
                        "append / truncate step")
    p.add_argument("--profile", action="store_true",
                   help="verify attention only: no clock sampling, sustained load, host-buffer pass, append "
                        "workload or CPU baseline (a short, repeatable run for ncu)")
    return p.parse_args(argv)


def measured_peaks():
    path = REPO / "MEASURED_PEAKS.json"
    if path.is_file():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profiled_traffic(name: str):
    """Per-launch DRAM bytes of the dominant kernel, transcribed from the
    committed ncu summary profiles/<name>.md (its line
    ``traffic_bytes_per_launch: N``, dram__bytes_read.sum +
    dram__bytes_write.sum of one captured launch), or None.  The figure is
    read from that file, not measured by this run: ncu cannot run inside the
    timed benchmark."""
    path = REPO / "profiles" / f"{name}.md"
    if not path.is_file():
        return None
    for line in path.read_text().splitlines():
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return int(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples while a region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu_index = gpu_index
        self.proc = None
        self.lines: list[tuple[float, str]] = []
        self._thread = None

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return
        self._thread = threading.Thread(target=self._read, daemon=True)
        self._thread.start()

    def _read(self) -> None:
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line.strip()))

    def stop(self) -> None:
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self._thread is not None:
            self._thread.join(timeout=5)

    def summary(self, t0: float, t1: float) -> dict:
        rows = []
        for ts, line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9 or not (t0 <= ts <= t1):
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, flags in rows for i, f in enumerate(flags) if f.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


def setup_distributed(args):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# ---------------------------------------------------------------------------
# verify attention (headline)
# ---------------------------------------------------------------------------

def verify_inputs(seed: int, rank: int = 0, world: int = 1):
    """Context lengths, a block table over a permuted pool, bf16-valued
    queries and the pool's block count for this rank's share of one global
    batch of ``32 * world`` sequences drawn from ``seed``, split over the
    ranks longest-first (balanced total context)."""
    import numpy as np

    rng = np.random.default_rng(seed)
    v = VERIFY
    lens = rng.integers(v["min_context"], v["max_context"] + 1, size=v["batch"] * world)
    if world > 1:
        from specdecode_b200.sharding import lpt_partition

        lens = lens[lpt_partition(lens.tolist(), world)[rank]]
        rng = np.random.default_rng([seed, rank])
    blocks = (lens + v["block_size"] - 1) // v["block_size"]
    nb = int(blocks.sum())
    perm = rng.permutation(nb)
    table = np.full((len(lens), int(blocks.max())), -1, dtype=np.int32)
    at = 0
    for b, n in enumerate(blocks):
        table[b, :n] = perm[at:at + n]
        at += n
    query = rng.standard_normal((len(lens), v["query_heads"], v["window"], v["head_dim"]), dtype=np.float32)
    return lens.astype(np.int64), table, nb, query


def build_verify(seed: int, device, rank: int = 0, world: int = 1):
    import torch

    from specdecode_b200.cuda_kv_cache import PagedVerifyAttention, attention_bytes
    from specdecode_b200.kv_cache import KVCacheConfig, PagedKVCache

    v = VERIFY
    lens, table, nb, query = verify_inputs(seed, rank, world)
    cache = PagedKVCache(KVCacheConfig(1, v["kv_heads"], v["head_dim"], block_size=v["block_size"], num_blocks=nb),
                         device=device, max_sequences=1, check_status=False)
    gen = torch.Generator(device=device).manual_seed(seed)
    # quantize N(0,1) K/V into every page with the append kernel, in slices
    cache.create_sequence("fill")
    tokens = nb * v["block_size"]
    step = 1 << 16
    for start in range(0, tokens, step):
        n = min(step, tokens - start)
        k = torch.randn((n, 1, v["kv_heads"], v["head_dim"]), generator=gen, device=device, dtype=torch.bfloat16)
        x = torch.randn((n, 1, v["kv_heads"], v["head_dim"]), generator=gen, device=device, dtype=torch.bfloat16)
        cache.append_tensor("fill", k, x)
    torch.cuda.synchronize()
    if cache.status_bits():
        raise RuntimeError("device fault while filling the benchmark pool")
    attention = PagedVerifyAttention.for_cache(cache)
    q = torch.from_numpy(query).to(torch.bfloat16).to(device)
    tables = torch.from_numpy(table).to(device)
    ctx = torch.from_numpy(lens.astype("int32")).to(device)
    nbytes = attention_bytes(lens.tolist(), v["query_heads"], v["kv_heads"], v["head_dim"], v["window"],
                             v["block_size"])
    return dict(cache=cache, attention=attention, q=q, tables=tables, ctx=ctx, max_len=int(lens.max()),
                bytes=nbytes, lens=lens, table=table, query=query)


def time_verify(state, steps: int, warmup: int, world: int, flush):
    import torch

    att, q, tables, ctx, max_len = state["attention"], state["q"], state["tables"], state["ctx"], state["max_len"]
    out = torch.empty_like(q)
    stream = torch.cuda.current_stream()
    for _ in range(warmup):
        flush.zero_()
        att(q, tables, ctx, max_len, 0, out=out)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    barrier(world)
    torch.cuda.synchronize()
    t_wall0 = time.monotonic()
    for i in range(steps):
        flush.zero_()
        hold_device()
        starts[i].record(stream)
        att(q, tables, ctx, max_len, 0, out=out)
        ends[i].record(stream)
    torch.cuda.synchronize()
    barrier(world)
    t_wall1 = time.monotonic()
    per = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    return sum(per), per, (t_wall0, t_wall1), out


def time_verify_e2e(state, steps: int, warmup: int, world: int, flush):
    """Host buffers in and out through the public attention API: every step
    copies its query from pinned host memory to the device, runs the
    attention and reads its output back into pinned host memory, all inside
    the timed region.  Steps are pipelined the way a serving loop would run
    them: step i + 1's query copy and step i - 1's output copy overlap step
    i's attention (three streams, two device and two host buffers each,
    ordered by events).  The timed region runs from before the first copy to
    after the last one; the pool is larger than L2, so no flush is needed
    between steps."""
    import torch

    att, tables, ctx, max_len = state["attention"], state["tables"], state["ctx"], state["max_len"]
    q_host = [state["q"].cpu().pin_memory() for _ in range(2)]
    out_host = [torch.empty_like(q_host[0]).pin_memory() for _ in range(2)]
    q_dev = [torch.empty_like(state["q"]) for _ in range(2)]
    out_dev = [torch.empty_like(state["q"]) for _ in range(2)]
    h2d, comp, d2h = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    Event = torch.cuda.Event
    done_in = [Event() for _ in range(2)]    # query buffer filled
    done_att = [Event() for _ in range(2)]   # attention finished with both buffers of the slot
    done_out = [Event() for _ in range(2)]   # output buffer read back
    used = [False, False]

    def run(n):
        for i in range(n):
            b = i & 1
            with torch.cuda.stream(h2d):
                if used[b]:
                    h2d.wait_event(done_att[b])
                q_dev[b].copy_(q_host[b], non_blocking=True)
                done_in[b].record(h2d)
            with torch.cuda.stream(comp):
                comp.wait_event(done_in[b])
                if used[b]:
                    comp.wait_event(done_out[b])
                att(q_dev[b], tables, ctx, max_len, 0, out=out_dev[b])
                done_att[b].record(comp)
            with torch.cuda.stream(d2h):
                d2h.wait_event(done_att[b])
                out_host[b].copy_(out_dev[b], non_blocking=True)
                done_out[b].record(d2h)
            used[b] = True

    run(warmup)
    torch.cuda.synchronize()
    barrier(world)
    start, end = Event(enable_timing=True), Event(enable_timing=True)
    start.record(h2d)
    run(steps)
    d2h.wait_stream(h2d)
    d2h.wait_stream(comp)
    end.record(d2h)
    torch.cuda.synchronize()
    barrier(world)
    return start.elapsed_time(end), q_host[0].numel() * q_host[0].element_size(), \
        out_host[0].numel() * out_host[0].element_size()


# ---------------------------------------------------------------------------
# end-to-end speculative decoding
# ---------------------------------------------------------------------------

def _random_llama(spec: dict, vocab: int, device):
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM

    config = LlamaConfig(hidden_size=spec["hidden"], intermediate_size=spec["intermediate"],
                         num_hidden_layers=spec["layers"], num_attention_heads=spec["heads"],
                         num_key_value_heads=spec["kv_heads"], head_dim=spec["head_dim"], vocab_size=vocab,
                         max_position_embeddings=8192, initializer_range=0.02)
    previous = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device(device):
            model = LlamaForCausalLM(config)
    finally:
        torch.set_default_dtype(previous)
    return model.eval()


def run_speculative(seed: int, device, world: int):
    """Batched speculative decoding through the paged caches: prefill the
    prompts, then time the decoding rounds (draft proposals, target verify,
    device-side acceptance, rollback) on the device; the attention calls of
    both models are timed individually."""
    import numpy as np
    import torch

    from specdecode_b200.kv_cache import KVCacheConfig, PagedKVCache
    from specdecode_b200.speculative import BatchedSpeculativeDecoder, DraftWindow

    sp = SPEC
    # start from an empty allocator cache: the earlier workloads leave large
    # cached blocks behind, and the decoding loop's own large tensors (the
    # rounds' probability rows) must not have to evict them mid-run
    gc.collect()
    torch.cuda.empty_cache()
    torch.manual_seed(seed)
    draft = _random_llama(sp["draft"], sp["vocab"], device)
    target = _random_llama(sp["target"], sp["vocab"], device)
    B = sp["batch"]
    # pool: every sequence at twice the new tokens on average; the block
    # tables allow the decoder's worst case for one sequence
    tokens = sp["prompt"] + 2 * sp["new_tokens"] + 2 * sp["max_window"]
    blocks = B * (-(-tokens // 16) + 1)

    def cache(spec):
        longest = sp["prompt"] + sp["new_tokens"] * (sp["max_window"] + 1) + 2 * sp["max_window"] + 2
        return PagedKVCache(KVCacheConfig(spec["layers"], spec["kv_heads"], spec["head_dim"], block_size=16,
                                          num_blocks=blocks), device=device, max_sequences=B, check_status=False,
                            max_blocks_per_sequence=-(-longest // 16) + 1)

    dec = BatchedSpeculativeDecoder(draft, target, cache(sp["draft"]), cache(sp["target"]),
                                    window=DraftWindow(sp["window"], sp["min_window"], sp["max_window"]),
                                    temperature=sp["temperature"], seed=seed, cuda_graphs=True)
    rng = np.random.default_rng(seed)
    prompts = torch.from_numpy(rng.integers(0, sp["vocab"], size=(B, sp["prompt"]), dtype=np.int64)).to(device)
    def timed_run():
        dec.window.size = sp["window"]
        # the decoding loop's host side allocates many small objects; collect
        # what earlier workloads left and freeze the survivors so that the
        # collector does not rescan them during the timed run
        gc.collect()
        gc.freeze()
        start, prefilled, end = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        barrier(world)
        torch.cuda.synchronize()
        start.record()
        result = dec.generate(prompts, sp["new_tokens"], prefill_done=prefilled)
        end.record()
        torch.cuda.synchronize()
        return result, start.elapsed_time(prefilled), prefilled.elapsed_time(end)

    with torch.no_grad():
        # decoding passes replayed from CUDA graphs: warm-up (eager first
        # passes, capture of the second), then the timed run
        dec.generate(prompts, 16)
        result, prefill_ms, decode_ms = timed_run()
        # the same run with eager passes and every attention call timed
        dec.cuda_graphs = False
        for session in (dec.draft, dec.target):
            session.timed = True
            session.timings.clear()
        eager_result, eager_prefill_ms, eager_decode_ms = timed_run()
        attn = {}
        for name, session in (("draft", dec.draft), ("target", dec.target)):
            ms, nbytes = session.attention_time()
            attn[name] = (ms, nbytes, len(session.timings))
            # once more, each attention call's launches queued behind a
            # device hold before its start event: device time per call
            session.timings.clear()
            session.timing_hold_cycles = HOLD_CYCLES
        timed_run()
    by_kind = {}
    for name, session in (("draft", dec.draft), ("target", dec.target)):
        for kind, (n, kms, kb) in session.attention_time_by_kind().items():
            by_kind[f"{name}_{kind}"] = {"calls": n, "ms": kms, "us_per_call": 1e3 * kms / n,
                                         "gbs": kb / (kms / 1e3) / 1e9 if kms > 0 else None}
        session.timed = False
        session.timing_hold_cycles = 0
    peak, peak_kind = measured_peaks()
    tokens_out = B * sp["new_tokens"]
    decode_max = max_over_ranks(decode_ms, world)
    eager_max = max_over_ranks(eager_decode_ms, world)
    attn_ms = sum(v[0] for v in attn.values())
    attn_bytes = sum(v[1] for v in attn.values())
    stats = result.stats
    out = {
        "config": f"draft Llama 16L d2048 32/8 heads D64, target Llama 32L d4096 32/8 heads D128, vocab "
                  f"{sp['vocab']}, random-init bf16 N(0, 0.02); batch {B} x prompt {sp['prompt']} uniform ids, "
                  f"{sp['new_tokens']} new tokens each, window {sp['min_window']}-{sp['max_window']} (start "
                  f"{sp['window']}), temperature {sp['temperature']}; both models attend over INT8 pages",
        "parallelism": f"request data-parallel x{world}, a full model pair per GPU",
        "tokens_per_s": sum_over_ranks(tokens_out, world) / (decode_max / 1e3),
        "tokens_per_s_with_prefill": sum_over_ranks(tokens_out, world) / (max_over_ranks(prefill_ms + decode_ms, world) / 1e3),
        "decode_ms": decode_max,
        "prefill_ms": max_over_ranks(prefill_ms, world),
        "decoding_passes": "CUDA graphs (draft steps and verify windows captured once, replayed)",
        "tokens_per_s_eager_passes": sum_over_ranks(tokens_out, world) / (eager_max / 1e3),
        "acceptance_rate": stats.acceptance_rate,
        "verification_rounds": stats.verification_rounds,
        "attention_ms_eager_run": attn_ms,
        "attention_share_of_eager_run": attn_ms / (eager_prefill_ms + eager_decode_ms),
        "attention_gbs": attn_bytes / (attn_ms / 1e3) / 1e9 if attn_ms > 0 else None,
        "attention_fraction_of_peak": attn_bytes / (attn_ms / 1e3) / 1e9 / peak if attn_ms > 0 else None,
        "attention_calls": {k: v[2] for k, v in attn.items()},
        # the eager run's attention calls by model and kind: prompt windows
        # ("prefill"), single-token draft steps ("decode"), target windows of
        # the proposals ("verify"); device time of each call (a rerun with a
        # device hold queued before every call's start event)
        "attention_by_kind": by_kind,
        "peak_source": peak_kind,
    }
    del dec, draft, target
    torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------
# append / rollback
# ---------------------------------------------------------------------------

def run_append(seed: int, device, steps: int, warmup: int, world: int, flush):
    import numpy as np
    import torch

    from specdecode_b200.kv_cache import KVCacheConfig, PagedKVCache

    a = APPEND
    rng = np.random.default_rng(seed + 1)
    order = rng.permutation(a["num_blocks"])
    cache = PagedKVCache(KVCacheConfig(a["layers"], a["kv_heads"], a["head_dim"], block_size=a["block_size"],
                                       num_blocks=a["num_blocks"]),
                         device=device, block_order=order, max_sequences=a["sequences"],
                         max_blocks_per_sequence=512, check_status=False)
    seqs = list(range(a["sequences"]))
    for s in seqs:
        cache.create_sequence(s)
    gen = torch.Generator(device=device).manual_seed(seed + 2)
    shape = (a["sequences"], a["window"], a["layers"], a["kv_heads"], a["head_dim"])
    factors = torch.exp(torch.empty((1, 1, 1, a["kv_heads"], 1), device=device).uniform_(
        math.log(0.1), math.log(10.0), generator=gen))
    keys = (torch.randn(shape, generator=gen, device=device) * factors).to(torch.bfloat16)
    values = (torch.randn(shape, generator=gen, device=device) * factors).to(torch.bfloat16)
    rolled = rng.integers(0, a["window"] + 1, size=(2 * (warmup + steps), a["sequences"]))
    spacer = flush[: 64 << 20]
    stream = torch.cuda.current_stream()
    append_ms, rollback_ms = [], []
    tokens_rolled = 0
    for i in range(warmup + steps):
        # host planning happens before the GPU is given a flush to chew on, so
        # the events below bracket device work only
        op = cache.prepare_append_batch(seqs, keys, values)
        flush.zero_()
        hold_device()
        e0, e1, e2, e3 = (torch.cuda.Event(enable_timing=True) for _ in range(4))
        e0.record(stream)
        cache.commit_append(op)
        e1.record(stream)
        counts = [cache.sequence_length(s) - int(r) for s, r in zip(seqs, rolled[i])]
        top = cache.prepare_truncate_batch(seqs, counts)
        spacer.zero_()
        hold_device()
        e2.record(stream)
        cache.commit_truncate(top)
        e3.record(stream)
        if i >= warmup:
            tokens_rolled += int(rolled[i].sum())
            append_ms.append((e0, e1))
            rollback_ms.append((e2, e3))
    torch.cuda.synchronize()
    # the same speculative step through the Python API, wall clock, no flushes
    torch.cuda.synchronize()
    h0 = time.perf_counter()
    for i in range(warmup + steps, warmup + 2 * steps):
        cache.append_batch(seqs, keys, values)
        counts = [cache.sequence_length(s) - int(r) for s, r in zip(seqs, rolled[i])]
        cache.truncate_batch(seqs, counts)
    torch.cuda.synchronize()
    host_s = time.perf_counter() - h0
    t_append = sum(s.elapsed_time(e) for s, e in append_ms)
    t_rollback = sum(s.elapsed_time(e) for s, e in rollback_ms)
    n_tokens = a["sequences"] * a["window"] * steps
    per_token = 2 * a["layers"] * a["kv_heads"] * a["head_dim"] * 2 + \
        2 * a["layers"] * a["kv_heads"] * a["head_dim"] + 2 * a["layers"] * a["kv_heads"] * 4
    per_rolled = 2 * a["layers"] * a["kv_heads"] * a["head_dim"] + 2 * a["layers"] * a["kv_heads"] * 4
    t_append = max_over_ranks(t_append, world)
    t_step = max_over_ranks(t_append + t_rollback, world)
    total_tokens = sum_over_ranks(n_tokens, world)
    result = {
        "config": "L32 Hkv8 D128 bf16, 256 sequences x 5-token window per step, 0-5 rolled back, "
                  "65536-block pool, randomized free list",
        "tokens_per_s": total_tokens / (t_append / 1e3),
        "step_tokens_per_s": total_tokens / (t_step / 1e3),
        "append_gbs": sum_over_ranks(n_tokens * per_token, world) / (t_append / 1e3) / 1e9,
        "rollback_gbs": (sum_over_ranks(tokens_rolled * per_rolled, world) / (t_rollback / 1e3) / 1e9)
        if t_rollback > 0 else None,
        "append_ms_per_step": t_append / steps,
        "rollback_ms_per_step": t_rollback / steps,
        "api_step_tokens_per_s": total_tokens / max_over_ranks(host_s + 1e-12, world),
        "algorithmic_bytes_per_token": per_token,
    }
    del cache, keys, values
    torch.cuda.empty_cache()
    return result


# ---------------------------------------------------------------------------
# CPU baseline (the reference's CPU path, bounded sample)
# ---------------------------------------------------------------------------

def profile_append(seed: int, device, steps: int) -> None:
    """The append / rollback step of the append workload on a small pool."""
    import numpy as np
    import torch

    from specdecode_b200.kv_cache import KVCacheConfig, PagedKVCache

    a = APPEND
    nb = 4096
    rng = np.random.default_rng(seed + 1)
    cache = PagedKVCache(KVCacheConfig(a["layers"], a["kv_heads"], a["head_dim"], block_size=a["block_size"],
                                       num_blocks=nb),
                         device=device, block_order=rng.permutation(nb), max_sequences=a["sequences"],
                         max_blocks_per_sequence=16, check_status=False)
    seqs = list(range(a["sequences"]))
    for s in seqs:
        cache.create_sequence(s)
    gen = torch.Generator(device=device).manual_seed(seed + 2)
    shape = (a["sequences"], a["window"], a["layers"], a["kv_heads"], a["head_dim"])
    factors = torch.exp(torch.empty((1, 1, 1, a["kv_heads"], 1), device=device).uniform_(
        math.log(0.1), math.log(10.0), generator=gen))
    keys = (torch.randn(shape, generator=gen, device=device) * factors).to(torch.bfloat16)
    values = (torch.randn(shape, generator=gen, device=device) * factors).to(torch.bfloat16)
    for _ in range(steps):
        cache.append_batch(seqs, keys, values)
        rolled = rng.integers(0, a["window"] + 1, size=a["sequences"])
        cache.truncate_batch(seqs, [cache.sequence_length(s) - int(r) for s, r in zip(seqs, rolled)])
    torch.cuda.synchronize()
    if cache.status_bits():
        raise RuntimeError("device fault in the append profile run")
    print(json.dumps({"profile_append": True, "steps": steps}))


def profile_case(name: str, seed: int, device, calls: int) -> None:
    """``calls`` untimed calls of one kernel family, then a fault check: the
    small, repeatable runs the ncu summaries are captured on."""
    import numpy as np
    import torch

    from specdecode_b200.cuda_kv_cache import PagedVerifyAttention
    from specdecode_b200.kv_cache import KVCacheConfig, PagedKVCache

    def filled_cache(lens, heads, dim, layers=1):
        nblk = (np.asarray(lens) + 15) // 16
        cache = PagedKVCache(KVCacheConfig(layers, heads, dim, block_size=16, num_blocks=int(nblk.sum())),
                             device=device, max_sequences=len(lens), check_status=False,
                             max_blocks_per_sequence=int(nblk.max()))
        gen = torch.Generator(device=device).manual_seed(seed)
        for b, T in enumerate(lens):
            cache.create_sequence(b)
            shape = (int(T), layers, heads, dim)
            cache.append_tensor(b, torch.randn(shape, generator=gen, device=device, dtype=torch.bfloat16),
                                torch.randn(shape, generator=gen, device=device, dtype=torch.bfloat16))
        return cache

    def attend(cache, lens, query_heads, windows):
        attention = PagedVerifyAttention.for_cache(cache)
        tables, ctx, max_len = cache.attention_inputs(list(range(len(lens))))
        gen = torch.Generator(device=device).manual_seed(seed + 1)
        queries = [torch.randn((len(lens), query_heads, window, cache.config.head_dim), generator=gen,
                               device=device).to(torch.bfloat16) for window in windows]
        for _ in range(calls):  # the windows interleaved: one launch of each per round
            for q in queries:
                attention(q, tables, ctx, max_len, 0)

    rng = np.random.default_rng(seed + 5)
    if name == "decode":
        lens = rng.integers(1024, 1177, size=64).tolist()
        for dim in (128, 64):
            cache = filled_cache(lens, 8, dim)
            attend(cache, lens, 32, (1, 6))
            torch.cuda.synchronize()
            if cache.status_bits():
                raise RuntimeError("device fault in the decode-shape profile run")
            del cache
    elif name == "simt":
        lens = rng.integers(1024, 4097, size=16).tolist()
        cache = filled_cache(lens, 8, 256)
        attend(cache, lens, 32, (5,))
        torch.cuda.synchronize()
        if cache.status_bits():
            raise RuntimeError("device fault in the CUDA-core attention profile run")
    elif name == "gather":
        state = build_verify(seed, device)
        slots = verify_slots(state, device)
        for _ in range(calls):
            state["cache"].gather_slots(slots, torch.bfloat16)
        torch.cuda.synchronize()
        if state["cache"].status_bits():
            raise RuntimeError("device fault in the gather profile run")
    elif name == "pages":
        run_device_pages(seed, device, max(1, calls // 2), max(1, calls - calls // 2), 1, num_blocks=4096)
    print(json.dumps({"profile_case": name, "calls": calls}))


def run_device_pages(seed: int, device, steps: int, warmup: int, world: int, num_blocks: int | None = None):
    """The append workload's speculative step (256 sequences append 5 tokens
    to 32 layers x 8 heads, then roll back 0-5 of them) with the block tables,
    lengths and free set on the device (DevicePagedCache): planning is a
    kernel, so the step is kernel launches only.  Wall-clock step rate through
    the Python API (as the append workload's api_step_tokens_per_s) and the
    step's device time."""
    import numpy as np
    import torch

    from specdecode_b200.device_pages import DevicePagedCache
    from specdecode_b200.kv_cache import KVCacheConfig

    a = APPEND
    rng = np.random.default_rng(seed + 1)
    nb = a["num_blocks"] if num_blocks is None else num_blocks
    cache = DevicePagedCache(KVCacheConfig(a["layers"], a["kv_heads"], a["head_dim"], block_size=a["block_size"],
                                           num_blocks=nb),
                             max_rows=a["sequences"], max_blocks_per_row=512,
                             block_order=rng.permutation(nb), device=device)
    rows = list(range(a["sequences"]))
    gen = torch.Generator(device=device).manual_seed(seed + 2)
    shape = (a["sequences"], a["window"], a["layers"], a["kv_heads"], a["head_dim"])
    keys = torch.randn(shape, generator=gen, device=device).to(torch.bfloat16)
    values = torch.randn(shape, generator=gen, device=device).to(torch.bfloat16)
    rolled = rng.integers(0, a["window"] + 1, size=(warmup + 2 * steps, a["sequences"]))

    def step(i):
        cache.append(rows, keys, values)
        cache.truncate(rows, [int(cache.length_bound[r]) - int(k) for r, k in zip(rows, rolled[i])])

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    h0 = time.perf_counter()
    for i in range(warmup, warmup + steps):
        step(i)
    torch.cuda.synchronize()
    host_s = time.perf_counter() - h0
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(HOLD_CYCLES * 5 * steps)  # the host queues every step before the start event runs
    start.record()
    for i in range(warmup + steps, warmup + 2 * steps):
        step(i)
    end.record()
    torch.cuda.synchronize()
    device_ms = start.elapsed_time(end) / steps
    cache.check_status()
    cache.validate_invariants()
    tokens = a["sequences"] * a["window"]
    del cache, keys, values
    torch.cuda.empty_cache()
    return {
        "workload": "256 sequences x 5 tokens appended then 0-5 rolled back per step, 32 layers x 8 heads x 128, "
                    "65536 blocks of 16, permuted block order; tables, lengths and free set on the device",
        "api_step_tokens_per_s": sum_over_ranks(tokens * steps, world) / max_over_ranks(host_s, world),
        "device_ms_per_step": max_over_ranks(device_ms, world),
        "device_step_tokens_per_s": sum_over_ranks(tokens, world) / (max_over_ranks(device_ms, world) / 1e3),
    }


SAMPLING = {"sequences": 64, "proposals": 6, "vocab": 128256}


def sampling_inputs(seed: int, device):
    """One verification round of the speculative workload's shape: float32
    softmax rows of the target (proposals + 1 per sequence) and of a draft
    whose logits are the target's plus N(0, 0.5) noise, proposals drawn from
    the draft, float64 uniforms."""
    import torch

    S, k, V = SAMPLING["sequences"], SAMPLING["proposals"], SAMPLING["vocab"]
    g = torch.Generator(device=device).manual_seed(seed + 7)
    logits = torch.randn((S, k + 1, V), generator=g, device=device) * 2.0
    target = torch.softmax(logits, dim=-1)
    draft = torch.softmax(logits[:, :k] + 0.5 * torch.randn((S, k, V), generator=g, device=device), dim=-1)
    tokens = torch.multinomial(draft.reshape(-1, V), 1, generator=g).view(S, k)
    uniforms = torch.rand((S, 2 * k + 1), generator=g, device=device, dtype=torch.float64)
    return target, draft, tokens, uniforms


def run_sampling(seed: int, device, steps: int, warmup: int, profile_only: bool = False):
    """Device acceptance and sampling at the speculative workload's shape:
    ``sdc_speculative_verify`` (acceptance probabilities of 64 x 6 proposals
    over 128 256 tokens, first rejection, correction or bonus sample) and the
    draft step's ``sdc_sample_categorical_rows`` over 64 rows.  Device time
    per call; the algorithmic bytes are every row each launch must read."""
    import torch

    from specdecode_b200.sampling import sample_rows, verify_batch

    target, draft, tokens, uniforms = sampling_inputs(seed, device)
    S, k, V = SAMPLING["sequences"], SAMPLING["proposals"], SAMPLING["vocab"]
    status = torch.zeros(1, dtype=torch.int32, device=device)
    draft_rows = target[:, 0].contiguous()

    def verify():
        return verify_batch(target, draft, tokens, uniforms[:, k:], status=status)

    def sample():
        return sample_rows(draft_rows, uniforms[:, 0], status=status)

    if profile_only:
        for _ in range(steps + warmup):
            verify()
            sample()
        torch.cuda.synchronize()
        if int(status.item()):
            raise RuntimeError("device fault in the sampling profile run")
        print(json.dumps({"profile_sampling": True, "rounds": steps + warmup}))
        return None

    def timed(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        # the Python wrappers take longer to launch than these kernels run:
        # hold the stream long enough (0.3 ms per call) for the host to queue
        # every timed call before the start event executes
        torch.cuda._sleep(HOLD_CYCLES * 3 * steps)
        start.record()
        for _ in range(steps):
            out = fn()
        end.record()
        torch.cuda.synchronize()
        return start.elapsed_time(end) / steps, out

    v_ms, (accepted, _, _) = timed(verify)
    s_ms, _ = timed(sample)
    if int(status.item()):
        raise RuntimeError(f"device fault bits 0x{int(status.item()):x} in the sampling workload")
    acc = accepted.cpu()
    rejected = int((acc < k).sum())
    # acceptance launch: every target and draft row of the proposals; the
    # deciding launch: the rejected pair of rows, or the bonus row
    v_bytes = 2 * k * S * V * 4 + (2 * rejected + (S - rejected)) * V * 4
    s_bytes = S * V * 4
    peak, peak_kind = measured_peaks()
    return {
        "workload": f"{S} sequences x {k} proposals, vocab {V}, float32 softmax rows",
        "verify_us": v_ms * 1e3,
        "verify_gbs": v_bytes / (v_ms / 1e3) / 1e9,
        "verify_frac": v_bytes / (v_ms / 1e3) / 1e9 / peak,
        "verify_bytes": v_bytes,
        "mean_accepted": float(acc.double().mean()),
        "sample_rows_us": s_ms * 1e3,
        "sample_rows_gbs": s_bytes / (s_ms / 1e3) / 1e9,
        "peak_gbs": peak,
        "peak_source": peak_kind,
    }


def verify_slots(state, device):
    """Physical slots of every cached token of the verify batch, sequence by
    sequence in context order (block table entry * block_size + offset): the
    token list a dequantize-then-attend caller gathers for one layer."""
    import numpy as np
    import torch

    bs = VERIFY["block_size"]
    parts = []
    for b, T in enumerate(state["lens"].tolist()):
        pos = np.arange(T, dtype=np.int64)
        parts.append(state["table"][b, pos // bs].astype(np.int64) * bs + pos % bs)
    return torch.from_numpy(np.concatenate(parts)).to(device)


def run_gather(state, device, steps: int, warmup: int, flush):
    """``sdc_gather_dequantize`` over the verify batch: every cached token of
    its 32 sequences (one layer, 8 KV heads x 128) dequantized to bf16, the
    reconstruct that a dequantize-then-attend path performs before its
    attention.  Device time per call, L2 flushed between calls; algorithmic
    bytes: per token and KV head the 2 x 128 codes and 2 scales read and the
    2 x 128 bf16 values written, plus the 8-byte slot."""
    import torch

    cache = state["cache"]
    slots = verify_slots(state, device)
    n = int(slots.numel())
    H, D = VERIFY["kv_heads"], VERIFY["head_dim"]
    out = (torch.empty((n, 1, H, D), dtype=torch.bfloat16, device=device),
           torch.empty((n, 1, H, D), dtype=torch.bfloat16, device=device))
    for _ in range(warmup):
        flush.zero_()
        cache.gather_slots(slots, torch.bfloat16, out=out)
    times = []
    for _ in range(steps):
        flush.zero_()
        hold_device()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        cache.gather_slots(slots, torch.bfloat16, out=out)
        end.record()
        times.append((start, end))
    torch.cuda.synchronize()
    if cache.status_bits():
        raise RuntimeError("device fault in the gather workload")
    ms = statistics.median(s.elapsed_time(e) for s, e in times)
    nbytes = n * (H * (2 * D + 8 + 2 * D * 2) + 8)
    peak, peak_kind = measured_peaks()
    gbs = nbytes / (ms / 1e3) / 1e9
    del out
    return {"workload": f"{n} cached tokens of the verify batch, one layer, 8 KV heads x 128, int8 pages -> bf16",
            "us_per_call": 1e3 * ms, "algorithmic_bytes": nbytes, "gbs": gbs,
            "frac_of_peak": gbs / peak if peak else None, "peak_source": peak_kind,
            "storage_synchronize": time_storage_sync(state)}


def time_storage_sync(state):
    """``CudaPagedKVCacheStorage.synchronize`` over the verify pool's one
    sequence (every cached page of the batch), wall clock: the first call
    binds all tokens, later ones find nothing changed.  The pages already
    live on the device, so a call is slot bookkeeping on the host; the
    reference's storage uploads its CPU-side cache instead."""
    from specdecode_b200.cuda_kv_cache import CudaPagedKVCacheStorage

    cache = state["cache"]

    class InlineRuntime:  # the runtime contract: run the transfer at once
        device = cache.device

        def submit_transfer(self, fn, *, wait_for=(), label=None):
            return fn()

    storage = CudaPagedKVCacheStorage(cache.config, InlineRuntime())
    tokens = cache.sequence_length("fill")
    t0 = time.perf_counter()
    storage.synchronize(cache, "fill")
    first = time.perf_counter() - t0
    t0 = time.perf_counter()
    for _ in range(5):
        storage.synchronize(cache, "fill")
    again = (time.perf_counter() - t0) / 5
    return {"tokens": tokens, "first_ms": 1e3 * first, "repeat_ms": 1e3 * again,
            "tokens_per_s": tokens / first}


def run_decode_shapes(seed: int, device, steps: int, warmup: int, flush):
    """Stand-alone attention calls at the end-to-end workload's shapes: 64
    sequences of about 1100 cached tokens, 32 query / 8 KV heads, a one-token
    decode step and a six-token verify window, head_dim 128 (the target)
    and 64 (the draft).  Device time per call with an L2 flush between
    calls: the figures the end-to-end loop's attention calls compare to."""
    import numpy as np
    import torch

    from specdecode_b200.cuda_kv_cache import PagedVerifyAttention, attention_bytes
    from specdecode_b200.kv_cache import KVCacheConfig, PagedKVCache

    B, Hq, Hkv, bs = 64, 32, 8, 16
    rng = np.random.default_rng(seed + 5)
    lens = rng.integers(1024, 1177, size=B)
    out = {}
    for D in (128, 64):
        nblk = (lens + bs - 1) // bs
        nb = int(nblk.sum())
        cache = PagedKVCache(KVCacheConfig(1, Hkv, D, block_size=bs, num_blocks=nb), device=device,
                             max_sequences=B, check_status=False, max_blocks_per_sequence=int(nblk.max()))
        gen = torch.Generator(device=device).manual_seed(seed + D)
        for b in range(B):
            cache.create_sequence(b)
            T = int(lens[b])
            cache.append_tensor(b, torch.randn((T, 1, Hkv, D), generator=gen, device=device, dtype=torch.bfloat16),
                                torch.randn((T, 1, Hkv, D), generator=gen, device=device, dtype=torch.bfloat16))
        attention = PagedVerifyAttention.for_cache(cache)
        tables, ctx, max_len = cache.attention_inputs(list(range(B)))
        for window in (1, 6):
            q = torch.randn((B, Hq, window, D), generator=gen, device=device).to(torch.bfloat16)
            res = torch.empty_like(q)
            for _ in range(warmup):
                flush.zero_()
                attention(q, tables, ctx, max_len, 0, out=res)
            times = []
            for _ in range(steps):
                flush.zero_()
                hold_device()
                start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record()
                attention(q, tables, ctx, max_len, 0, out=res)
                end.record()
                times.append((start, end))
            torch.cuda.synchronize()
            ms = statistics.median(s.elapsed_time(e) for s, e in times)
            nbytes = attention_bytes(lens.tolist(), Hq, Hkv, D, window, bs)
            out[f"d{D}_window{window}"] = {"us_per_call": 1e3 * ms, "gbs": nbytes / (ms / 1e3) / 1e9}
        if cache.status_bits():
            raise RuntimeError("device fault in the decode-shape workload")
        del cache, attention
        torch.cuda.empty_cache()
    out["workload"] = ("64 sequences x 1024-1176 cached tokens, 32 query / 8 KV heads, block 16, one layer; "
                       "median of the timed calls, L2 flushed between calls")
    return out


def run_long_context(seed: int, rank: int, world: int, device, steps: int, warmup: int):
    """Llama-3.1-70B long-context verify, one layer: 8 sequences x 131072
    tokens, 64 query / 8 KV heads, window 5.  KV heads are split over the
    ranks (tensor parallel); each rank holds its heads' pages of every
    sequence and the outputs are all-gathered over NCCL.  Strong scaling:
    the total work is fixed."""
    import numpy as np
    import torch

    from specdecode_b200.cuda_kv_cache import PagedVerifyAttention, attention_bytes
    from specdecode_b200.kv_cache import KVCacheConfig, PagedKVCache
    from specdecode_b200.sharding import PeerHeadGather, TensorParallelVerifyAttention, head_shard, shard_query

    c = LONG
    shard = head_shard(rank, world, c["kv_heads"], c["query_heads"])
    B, T, bs, D, kw = c["batch"], c["context"], c["block_size"], c["head_dim"], c["window"]
    per_seq = T // bs
    nb = B * per_seq
    cache = PagedKVCache(KVCacheConfig(1, shard.kv_per_rank, D, block_size=bs, num_blocks=nb), device=device,
                         max_sequences=1, check_status=False)
    gen = torch.Generator(device=device).manual_seed(seed + 17 * rank)
    cache.create_sequence("fill")
    step = 1 << 16
    for start in range(0, nb * bs, step):
        n = min(step, nb * bs - start)
        k = torch.randn((n, 1, shard.kv_per_rank, D), generator=gen, device=device, dtype=torch.bfloat16)
        v = torch.randn((n, 1, shard.kv_per_rank, D), generator=gen, device=device, dtype=torch.bfloat16)
        cache.append_tensor("fill", k, v)
    torch.cuda.synchronize()
    rng = np.random.default_rng(seed)  # the same tables and queries on every rank
    tables = torch.from_numpy(rng.permutation(nb).astype(np.int32).reshape(B, per_seq)).to(device)
    lens = torch.full((B,), T, dtype=torch.int32, device=device)
    query = torch.from_numpy(rng.standard_normal((B, c["query_heads"], kw, D), dtype=np.float32)).to(
        torch.bfloat16).to(device)
    attention = PagedVerifyAttention.for_cache(cache)
    tp = TensorParallelVerifyAttention(attention, shard)
    q_local = shard_query(query, shard).contiguous()
    out_local = torch.empty_like(q_local)
    stream = torch.cuda.current_stream()

    def timed(fn):
        for _ in range(warmup):
            fn()
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        barrier(world)
        torch.cuda.synchronize()
        for i in range(steps):
            hold_device()
            starts[i].record(stream)
            fn()
            ends[i].record(stream)
        torch.cuda.synchronize()
        barrier(world)
        return max_over_ranks(sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / steps, world)

    local_ms = timed(lambda: attention(q_local, tables, lens, T, 0, out=out_local))
    full_ms = timed(lambda: tp(query, tables, lens, T, 0))
    peer_ms = None
    if world > 1:
        # the all-gather fused into the attention's output stores (peer
        # stores over NVLink + bounded flag waits), against the NCCL one
        gather = PeerHeadGather(cache, shard, B, kw)
        try:
            peer_ms = timed(lambda: gather(query, tables, lens, T, 0))
            if not torch.equal(gather(query, tables, lens, T, 0), tp(query, tables, lens, T, 0)):
                raise RuntimeError("the fused head gather and the NCCL all-gather disagree")
        finally:
            gather.close()
    if cache.status_bits():
        raise RuntimeError(f"device fault bits 0x{cache.status_bits():x} in the long-context benchmark")
    per_rank = attention_bytes([T] * B, shard.q_per_rank, shard.kv_per_rank, D, kw, bs)
    total = sum_over_ranks(per_rank, world)
    shard_local = None
    if world == 1:
        del cache, attention, tp
        torch.cuda.empty_cache()
        shard_local = long_context_shards(seed, device, steps, warmup)
    return {
        "config": "70B long-context verify, one layer: B8 x 131072 tokens, Hq64 Hkv8 D128 window5 bs16, "
                  "randomly permuted blocks",
        "parallelism": f"KV-head tensor-parallel x{world}" + (
            "; outputs gathered by NCCL all-gather, or by the attention's own peer stores + flags (fused)"
            if world > 1 else ""),
        "scaling": "strong",
        "gbs": total / (local_ms / 1e3) / 1e9,
        "ms_per_step": local_ms,
        "gbs_with_allgather": total / (full_ms / 1e3) / 1e9,
        "ms_per_step_with_allgather": full_ms,
        "gbs_with_fused_gather": total / (peer_ms / 1e3) / 1e9 if peer_ms else None,
        "ms_per_step_with_fused_gather": peer_ms,
        "allgather_bytes": B * c["query_heads"] * kw * D * 2 if world > 1 else 0,
        "algorithmic_bytes_per_step": total,
        "shard_local": shard_local,
    }


def long_context_shards(seed: int, device, steps: int, warmup: int):
    """Rank 0's local attention in the long-context workload split over 2, 4
    and 8 ranks, timed on this one GPU (its pages only: Hkv/G KV heads of
    every sequence): how the per-GPU rate holds as the shard shrinks."""
    import numpy as np
    import torch

    from specdecode_b200.cuda_kv_cache import PagedVerifyAttention, attention_bytes
    from specdecode_b200.kv_cache import KVCacheConfig, PagedKVCache
    from specdecode_b200.sharding import head_shard, shard_query

    c = LONG
    B, T, bs, D, kw = c["batch"], c["context"], c["block_size"], c["head_dim"], c["window"]
    per_seq = T // bs
    nb = B * per_seq
    out = {}
    for world in (2, 4, 8):
        shard = head_shard(0, world, c["kv_heads"], c["query_heads"])
        cache = PagedKVCache(KVCacheConfig(1, shard.kv_per_rank, D, block_size=bs, num_blocks=nb), device=device,
                             max_sequences=1, check_status=False)
        gen = torch.Generator(device=device).manual_seed(seed + world)
        cache.create_sequence("fill")
        for start in range(0, nb * bs, 1 << 16):
            n = min(1 << 16, nb * bs - start)
            k = torch.randn((n, 1, shard.kv_per_rank, D), generator=gen, device=device, dtype=torch.bfloat16)
            v = torch.randn((n, 1, shard.kv_per_rank, D), generator=gen, device=device, dtype=torch.bfloat16)
            cache.append_tensor("fill", k, v)
        rng = np.random.default_rng(seed)
        tables = torch.from_numpy(rng.permutation(nb).astype(np.int32).reshape(B, per_seq)).to(device)
        lens = torch.full((B,), T, dtype=torch.int32, device=device)
        query = torch.from_numpy(rng.standard_normal((B, c["query_heads"], kw, D), dtype=np.float32)).to(
            torch.bfloat16).to(device)
        q_local = shard_query(query, shard).contiguous()
        attention = PagedVerifyAttention.for_cache(cache)
        res = torch.empty_like(q_local)
        for _ in range(warmup):
            attention(q_local, tables, lens, T, 0, out=res)
        times = []
        for _ in range(steps):
            hold_device()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            attention(q_local, tables, lens, T, 0, out=res)
            end.record()
            times.append((start, end))
        torch.cuda.synchronize()
        if cache.status_bits():
            raise RuntimeError("device fault in the long-context shard timing")
        ms = statistics.median(s.elapsed_time(e) for s, e in times)
        nbytes = attention_bytes([T] * B, shard.q_per_rank, shard.kv_per_rank, D, kw, bs)
        out[f"ranks{world}"] = {"kv_heads": shard.kv_per_rank, "ms": ms, "gbs": nbytes / (ms / 1e3) / 1e9}
        del cache, attention
        torch.cuda.empty_cache()
    return out


def verify_seq_bytes(lens):
    """Algorithmic bytes of each sequence's share of a verify-attention call:
    its cached tokens' INT8 key / value codes and fp32 scales for every KV
    head, its bf16 query and output rows and its block-table entries (their
    sum over a batch is ``attention_bytes``)."""
    v = VERIFY
    per_token = 2 * v["kv_heads"] * v["head_dim"] + 2 * v["kv_heads"] * 4
    rows = v["query_heads"] * v["window"] * v["head_dim"] * 2
    return [int(T) * per_token + 2 * rows + -(-int(T) // v["block_size"]) * 4 for T in lens]


def config1_events(seed: int, only=None):
    """The reference's CPU-runnable workload: ``("append", seq, keys,
    values)`` with float32 N(0,1) ``[tokens, 16, 8, 64]`` arrays and
    ``("truncate", seq, new_length)``.  Every sequence prefills 512 tokens;
    then each of 64 rounds appends a 5-token window to every sequence and
    keeps the prefix accepted by Bernoulli(0.7) draws up to the first
    rejection.  ``only``: yield just that sequence's events (the draws are
    the same as for the whole workload)."""

    for event in _config1_all(seed):
        if only is None or event[1] == only:
            yield event


def _config1_all(seed: int):
    import numpy as np

    c = CONFIG1
    rng = np.random.default_rng(seed)
    dims = (c["layers"], c["kv_heads"], c["head_dim"])
    lengths = [0] * c["sequences"]
    for s in range(c["sequences"]):
        yield ("append", s, rng.standard_normal((c["prefill"], *dims), dtype=np.float32),
               rng.standard_normal((c["prefill"], *dims), dtype=np.float32))
        lengths[s] = c["prefill"]
    for _ in range(c["rounds"]):
        for s in range(c["sequences"]):
            yield ("append", s, rng.standard_normal((c["window"], *dims), dtype=np.float32),
                   rng.standard_normal((c["window"], *dims), dtype=np.float32))
            accepted = 0
            while accepted < c["window"] and rng.random() < c["accept_p"]:
                accepted += 1
            lengths[s] += accepted
            yield ("truncate", s, lengths[s])


def append_events(seed: int, sequences: int, steps: int):
    """The append workload's speculative step for ``sequences`` of its
    sequences: each step appends a 5-token window of bf16-valued N(0,1) keys
    and values (32 layers x 8 heads x 128, scaled by per-head factors
    log-uniform in [0.1, 10]) to every sequence, then rolls 0-5 tokens back."""
    import numpy as np
    import torch

    a = APPEND
    rng = np.random.default_rng(seed)
    factors = np.exp(rng.uniform(math.log(0.1), math.log(10.0), size=(1, 1, a["kv_heads"], 1)))
    dims = (a["window"], a["layers"], a["kv_heads"], a["head_dim"])

    def draw():
        x = (rng.standard_normal(dims) * factors).astype(np.float32)
        return torch.from_numpy(x).to(torch.bfloat16).float().numpy()

    lengths = [0] * sequences
    for _ in range(steps):
        for s in range(sequences):
            yield ("append", s, draw(), draw())
            lengths[s] += a["window"]
        for s in range(sequences):
            lengths[s] -= int(rng.integers(0, a["window"] + 1))
            yield ("truncate", s, lengths[s])


def cpu_reference_attention(lens, table, query, pool, *, budget_s: float, min_passes: int = 1):
    """The reference's own paged attention on the host cores (CPU baseline
    leg (i)): ``submit_paged_attention`` unchanged, one call per sequence."""
    from oracle import reference_runs as rr

    order, seconds, _ = rr.time_submit_paged_attention(pool, lens, table, query, VERIFY["block_size"], budget_s,
                                                       min_passes=min_passes)
    per = verify_seq_bytes(lens)
    t = sum(seconds)
    passes = len(order) / len(lens)
    return {"value": sum(per[b] for b in order) / t / 1e9, "unit": "GB/s", "cores": rr.host_threads(),
            "kind": "reference",
            "sample": f"the reference's submit_paged_attention (src/specdecode/cuda_kv_cache.py:370-503, unchanged, "
                      f"imported from oracle/_ref) on CPU torch through an inline runtime shim, one call per "
                      f"sequence (its API is batch 1): {len(order)} calls = {passes:.2f} passes over the "
                      f"{len(lens)} sequences ({sum(int(lens[b]) for b in order)} cached tokens), {t:.1f} s",
            "ms_per_pass": 1e3 * t / passes}


def cpu_reference_reconstruct(lens, query, *, budget_s: float, seed: int):
    """CPU baseline leg (ii): the reference's CPU reconstruct path, the
    native dequantization plus Python reconstruction of
    ``materialize_legacy_cache`` and torch CPU SDPA."""
    from oracle import reference_runs as rr

    v = VERIFY
    r = rr.time_reconstruct_attention(lens, query, v["kv_heads"], v["head_dim"], v["block_size"], budget_s, seed)
    n = r["sequences"]
    return {"value": sum(verify_seq_bytes(lens[:n])) / r["seconds"] / 1e9, "unit": "GB/s", "cores": r["threads"],
            "kind": "reference",
            "sample": f"the reference's HuggingFacePagedCacheMirror.materialize_legacy_cache "
                      f"(src/specdecode/hf_paged_cache.py:247-313: NativeKVQuantizer dequantization over the "
                      f"reference's library, Python reconstruction) + GQA expansion + torch CPU SDPA in bf16, "
                      f"first {n} of {len(lens)} sequences ({r['tokens']} cached tokens), {r['seconds']:.1f} s",
            "synchronize_tokens_per_s": r["tokens"] / r["synchronize_seconds"]}


def cpu_reference_append(events, shape: dict, *, budget_s: float, what: str):
    """The reference's ``PagedKVCache.append_many`` / ``truncate`` with its
    ``NativeKVQuantizer`` over ``events`` until ``budget_s`` of timed work."""
    from oracle import reference_runs as rr

    r = rr.time_append_rollback(shape["layers"], shape["kv_heads"], shape["head_dim"], shape["block_size"],
                                shape["num_blocks"], events, budget_s)
    return {"value": r["appended_tokens"] / r["append_seconds"], "unit": "tokens/s", "cores": 1,
            "kind": "reference",
            "rollback_tokens_per_s": r["rolled_back_tokens"] / r["truncate_seconds"] if r["truncate_seconds"] else None,
            "sample": f"the reference's PagedKVCache.append_many + truncate (src/specdecode/kv_cache.py:290-336, "
                      f":395-420) with NativeKVQuantizer over the reference's library, one Python thread: {what}, "
                      f"{r['events']} calls over {r['sequences']} sequences, {r['appended_tokens']} tokens appended "
                      f"in {r['append_seconds']:.1f} s, {r['rolled_back_tokens']} rolled back in "
                      f"{r['truncate_seconds']:.2f} s"}


def run_config1(seed: int, device, repeats: int = 3):
    """The reference's CPU-runnable workload through this library's
    ``PagedKVCache`` on the GPU: every append copies its float32 keys and
    values from pinned host memory, every rollback is kernel (b).  Wall time
    of the whole workload through the Python API, best of ``repeats`` runs
    after one warm-up run, each on a fresh cache."""
    import torch

    from specdecode_b200.kv_cache import KVCacheConfig, PagedKVCache

    c = CONFIG1
    events = []
    appended = rolled = h2d = 0
    lengths = [0] * c["sequences"]
    for e in config1_events(seed):
        if e[0] == "append":
            k, v = torch.from_numpy(e[2]).pin_memory(), torch.from_numpy(e[3]).pin_memory()
            events.append(("append", e[1], k, v))
            appended += k.shape[0]
            lengths[e[1]] += k.shape[0]
            h2d += 2 * k.numel() * k.element_size()
        else:
            rolled += lengths[e[1]] - e[2]
            lengths[e[1]] = e[2]
            events.append(e)

    def once():
        cache = PagedKVCache(KVCacheConfig(c["layers"], c["kv_heads"], c["head_dim"], block_size=c["block_size"],
                                           num_blocks=c["num_blocks"]), device=device, check_status=False)
        for s in range(c["sequences"]):
            cache.create_sequence(s)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for e in events:
            if e[0] == "append":
                cache.append_tensor(e[1], e[2], e[3])
            else:
                cache.truncate(e[1], e[2])
        torch.cuda.synchronize()
        t = time.perf_counter() - t0
        if cache.status_bits():
            raise RuntimeError("device fault in the CPU-runnable workload")
        return t

    once()
    t = min(once() for _ in range(repeats))
    return {"workload": "L16 Hkv8 D64 bs16, 4096 blocks, fp32 N(0,1) keys/values from pinned host memory: 4 sequences "
                        "prefill 512 tokens, 64 rounds append a 5-token window each and roll back past the first "
                        "Bernoulli(0.7) rejection",
            "appended_tokens": appended, "rolled_back_tokens": rolled, "seconds": t,
            "tokens_per_s": appended / t, "h2d_bytes": h2d}


def run_reference_arm(args, rank: int, world: int) -> None:
    """The reference's own CPU path on this host's cores, never this
    library: the config-2 pool is quantized by the oracle's C restatement of
    the reference rule and the timed calls are the reference's code from
    oracle/_ref.  Rank 0 alone runs; other ranks return at once."""
    if rank != 0:
        return
    from oracle import reference_runs as rr

    try:
        rr.reference_package()
    except rr.ReferenceUnavailable as error:
        print(json.dumps({"impl": "reference", "unavailable": str(error)}))
        return
    v = VERIFY
    lens, table, nb, query = verify_inputs(args.seed)
    pool = rr.verify_pool(nb, v["kv_heads"], v["head_dim"], v["block_size"], args.seed)
    # warm-up passes, then K timed passes (one step = one pass over the batch),
    # fewer if a pass is slow enough that K would exceed about a minute
    warm = cpu_reference_attention(lens, table, query, pool, budget_s=0.0, min_passes=1)
    for _ in range(min(args.warmup, 3) - 1):
        cpu_reference_attention(lens, table, query, pool, budget_s=0.0, min_passes=1)
    passes = max(1, min(args.steps, int(60.0 / max(warm["ms_per_pass"] / 1e3, 1e-3))))
    base = cpu_reference_attention(lens, table, query, pool, budget_s=0.0, min_passes=passes)
    reconstruct = cpu_reference_reconstruct(lens, query, budget_s=6.0, seed=args.seed + 7)
    append = cpu_reference_append(append_events(args.seed + 1, 4, 1000), APPEND, budget_s=8.0,
                                  what="the append workload's step for 4 of its 256 sequences")
    config1 = cpu_reference_append(config1_events(args.seed, only=0), CONFIG1, budget_s=10.0,
                                   what="sequence 0 of the CPU-runnable workload's 4 (prefill, then its rounds)")
    line = {
        "impl": "reference", "metric": METRIC, "value": base["value"], "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "passes_timed": passes, "ms_per_step": base["ms_per_pass"],
        "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) bf16 K/V quantized to INT8 pages, N(0,1) bf16 queries)",
        "config": {"workload": VERIFY_WORKLOAD},
        "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": base["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "reconstruct_path": reconstruct,
        "append": append,
        "config1": config1,
    }
    print(json.dumps(line))


def main(argv=None) -> int:
    args = parse_args(argv)
    if args.steps < 1 or args.warmup < 3:
        raise SystemExit("need --steps >= 1 and --warmup >= 3")
    rank, world, local = setup_distributed(args)
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return 0

    import torch

    device = torch.device("cuda", local)
    if args.profile_append:
        profile_append(args.seed, device, args.steps + args.warmup)
        return 0
    if args.profile_sampling:
        run_sampling(args.seed, device, args.steps, args.warmup, profile_only=True)
        return 0
    if args.profile_case:
        profile_case(args.profile_case, args.seed, device, args.steps + args.warmup)
        return 0
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=device)
    state = build_verify(args.seed, device, rank, world)

    if args.profile:
        t_ms, _, _, _ = time_verify(state, args.steps, args.warmup, world, flush)
        if state["cache"].status_bits():
            raise RuntimeError("device fault in the verify benchmark")
        if rank == 0:
            print(json.dumps({"profile_run": True, "ms_per_step": t_ms / args.steps,
                              "gbs": state["bytes"] / (t_ms / args.steps / 1e3) / 1e9}))
        return 0
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler is not None:
        sampler.start()
        time.sleep(0.3)
    # sustained load around the timed region so the sampler sees the kernel's clocks
    sustain_until = time.monotonic() + 1.0
    while time.monotonic() < sustain_until:
        state["attention"](state["q"], state["tables"], state["ctx"], state["max_len"], 0)
        torch.cuda.synchronize()
    t_ms, per, (w0, w1), out = time_verify(state, args.steps, args.warmup, world, flush)
    if sampler is not None:
        time.sleep(0.2)
        sampler.stop()
    bits = state["cache"].status_bits()
    if bits:
        raise RuntimeError(f"device fault bits 0x{bits:x} in the verify benchmark")
    t_max = max_over_ranks(t_ms, world)
    total_bytes = sum_over_ranks(state["bytes"] * args.steps, world)
    value = total_bytes / (t_max / 1e3) / 1e9
    peak, peak_kind = measured_peaks()
    per_launch_ms = t_ms / args.steps
    achieved = state["bytes"] / (per_launch_ms / 1e3) / 1e9

    e2e_ms, h2d, d2h = time_verify_e2e(state, args.steps, args.warmup, world, flush)
    e2e_value = total_bytes / (max_over_ranks(e2e_ms, world) / 1e3) / 1e9
    gather = run_gather(state, device, args.steps, args.warmup, flush)

    append = None
    if not args.skip_append:
        append = run_append(args.seed + 1000 * rank, device, args.steps, args.warmup, world, flush)

    long_ctx = None
    if not args.skip_long:
        long_ctx = run_long_context(args.seed, rank, world, device, args.steps, args.warmup)

    decode_shapes = None
    if not args.skip_speculative:
        decode_shapes = run_decode_shapes(args.seed + 1000 * rank, device, args.steps, args.warmup, flush)

    device_pages = None
    if not args.skip_device_pages:
        device_pages = run_device_pages(args.seed + 1000 * rank, device, args.steps, args.warmup, world)

    sampling = None
    if not args.skip_sampling:
        sampling = run_sampling(args.seed + 1000 * rank, device, args.steps, args.warmup)

    speculative = None
    if not args.skip_speculative:
        speculative = run_speculative(args.seed + 1000 * rank, device, world)

    cpu = config1 = None
    if not args.skip_config1:
        config1 = run_config1(args.seed + 1000 * rank, device)
    if rank == 0 and world == 1 and not args.skip_cpu_baseline:
        # the reference's own CPU path on this host, bounded samples of the
        # same workloads (the attention leg reads this run's pool)
        cache = state["cache"]
        pool = {"keys": cache.keys_view[:, :, :1].contiguous().cpu().numpy(),
                "values": cache.values_view[:, :, :1].contiguous().cpu().numpy(),
                "key_scales": cache.key_scales_view[:, :, :1].contiguous().cpu().numpy(),
                "value_scales": cache.value_scales_view[:, :, :1].contiguous().cpu().numpy()}
        cpu = cpu_reference_attention(state["lens"], state["table"], state["query"], pool, budget_s=3.0)
        del pool
        cpu["reconstruct_path"] = cpu_reference_reconstruct(state["lens"], state["query"], budget_s=4.0,
                                                            seed=args.seed + 7)
        if append is not None:
            append["cpu_baseline"] = cpu_reference_append(
                append_events(args.seed + 1, 4, 1000), APPEND, budget_s=6.0,
                what="the append workload's step for 4 of its 256 sequences")
        if config1 is not None:
            config1["cpu_baseline"] = cpu_reference_append(
                config1_events(args.seed, only=0), CONFIG1, budget_s=8.0,
                what="sequence 0 of the CPU-runnable workload's 4 (prefill, then its rounds)")

    clocks = sampler.summary(w0 - 1.2, w1 + 0.1) if sampler is not None else None
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": t_max / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "int8 pages, fp32 softmax/accumulate",
            "data": "synthetic (seeded N(0,1) bf16 K/V quantized to INT8 pages, N(0,1) bf16 queries)",
            "config": {
                "workload": VERIFY_WORKLOAD,
                "global_batch": VERIFY["batch"] * world,
                "parallelism": f"request data-parallel x{world} (no collective): one batch of "
                               f"{VERIFY['batch'] * world} sequences split over the ranks longest-first",
                "l2": "256 MiB flush between timed iterations; pool larger than L2",
            },
            "fraction_of_peak": value / world / peak,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_source": peak_kind,
                         "traffic": profiled_traffic("verify_attention_8b"),
                         "algorithmic_bytes_per_launch": state["bytes"]},
            "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": 3 * args.steps,
            "append": append,
            "config1": config1,
            "long_context_70b": long_ctx,
            "device_pages": device_pages,
            "speculative_sampling": sampling,
            "speculative_e2e": speculative,
            "decode_shapes": decode_shapes,
            "gather_dequantize": gather,
            "cpu_baseline": cpu,
            "clocks": clocks,
        }
        print(json.dumps(line))
    if world > 1:
        import torch.distributed as dist

        barrier(world)
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
