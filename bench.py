"""Quest sparse-decode benchmark (benchmark config 1) — one JSON line on rank 0.

Workload (per GPU): 64 requests, each with a 32 768-token prefix (512 complete
pages of 64), Qwen3-30B-A3B attention geometry (32 query / 4 KV heads,
head_dim 128, bf16), 48 layers, Quest top_k 2048 (31 pages + recent 64).  A
*step* is one decode step through the drop-in backend's public interface:
``init_forward_metadata`` (bounds fold of the previous token for all 48
layers) then ``forward`` for each of the 48 layers (new K/V write + GQA mean
+ page scores + top-k + req_to_token translation + split-K sparse
attention).  Unit: layer-steps/s, a layer-step being one layer of decode for
the whole 64-request batch; whole-job value = sum over ranks.

The full KV of 48 layers x 64 x 32 768 tokens (206 GB) does not fit one
B200, so ``RESIDENT`` physical KV buffers are aliased over the 48 layers
(layer l reads buffer l % RESIDENT); Quest bounds are kept for all 48 layers.
Every layer-step reads ~338 MB of distinct data (far beyond the 126 MB L2),
so aliasing changes no byte counts.  Inputs are synthetic (seeded N(0,1)
scaled per channel by LogNormal(0, 0.5)); no dataset exists for this path.

``--impl reference`` times the reference's own ``QuestOnlyBackend`` (torch on
the host cores, CPU pools) on config 1's 64-request batch, one layer per step
(a layer-step), with the numpy restatement under ``oracle/`` reported beside
it; the GPU arm's ``cpu_baseline`` is the same measurement.

Other single-GPU cases, each printing its own JSON line (not the headline):
``--case config0`` (one 8K-token request, one layer: microseconds per
layer-step), ``--case prefill`` (one 32K-token prefill's K/V write + Quest
bounds over 48 layers, fused against the reference's order), ``--case config2`` (16 ragged
requests up to 131K tokens, Mode 2) and ``--case config3`` (HiSparse, 32
requests at 65,536 tokens with the host tier, against the host-link
roofline), ``--case config4`` (one GPU's 8-request shard of the end-to-end
run: the reference ``Engine`` and random-init Qwen3-30B-A3B with the B200
attention backend; decode tokens/s and the backend's share of it),
``--case prefill_attn`` (the dense causal prefill attention of one 32K-token
request on the tensor cores, TFLOP/s against the reference's gather + SDPA),
``--case moe`` (one Qwen3-30B-A3B MoE block at 8 decode tokens and a 32K-token
prefill, against the reference's per-expert loop).
``--context-limit`` runs config 1 under a larger engine ``max_context_len``.
Multi-GPU: one process per GPU (torchrun); config 1's 64 requests are sharded
in contiguous blocks over the GPUs (64/N per GPU) with no collective on the
hot path (strong scaling, the configuration the benchmark names); ``--weak``
gives every GPU its own 64 requests instead.
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
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
from tests._reference import ensure_importable  # noqa: E402  (the backends plug into the reference package)

ensure_importable()

H, KV, D = 32, 4, 128
TOP_K, PAGE = 2048, 64
LAYERS = 48
N_REQ = 64
PREFIX = 32768
RESIDENT = 4
METRIC = "Quest sparse-decode layer-steps/sec per GPU and box"
UNIT = "layer-steps/s"

# bytes per request-layer of the long-request layer step (algorithmic):
# q 8192 + new K/V 2048 + bounds append 4096 + positions 8192 + req_to_token 8192
# + K/V gather 2048 rows x 2048 B + output 8192, plus 2048 B per candidate page
BYTES_FIXED = 8192 + 2048 + 4096 + 8192 + 8192 + 2048 * 2048 + 8192
ATTN_BYTES_PER_REQ = 8192 + 8192 + 2048 * 2048 + 8192  # q + rows + K/V rows + out


def layer_step_bytes(candidate_pages: int, n_req: int = N_REQ) -> int:
    return n_req * (BYTES_FIXED + 2048 * candidate_pages)


# --------------------------------------------------------------------------- clocks


class ClockSampler:
    """Samples nvidia-smi clocks / throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()

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
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(smax) if smax else None,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


# --------------------------------------------------------------------------- setup


class _Pool:
    """``MHATokenToKVPool`` whose 48 layer buffers alias ``RESIDENT`` physical ones."""

    def __init__(self, k_phys, v_phys, layers):
        self.k_buffer = [k_phys[i % len(k_phys)] for i in range(layers)]
        self.v_buffer = [v_phys[i % len(v_phys)] for i in range(layers)]
        self.num_layers = layers
        self.kv_heads, self.head_dim = KV, D
        self.dtype = torch.bfloat16
        self.device = k_phys[0].device
        self.size = k_phys[0].shape[0] - 1

    def get_key_buffer(self, i):
        return self.k_buffer[i]

    def get_value_buffer(self, i):
        return self.v_buffer[i]

    def get_kv_buffer(self, i):
        return self.k_buffer[i], self.v_buffer[i]

    def set_kv_buffer(self, i, loc, k, v):
        self.k_buffer[i][loc.long()] = k.to(self.dtype)
        self.v_buffer[i][loc.long()] = v.to(self.dtype)


def build_config1(dev, total_steps: int, seed: int, n_req: int = N_REQ, prefix: int = PREFIX,
                  layers: int = LAYERS, resident: int = RESIDENT, context_limit: int | None = None):
    from qwenquest_b200.backends import B200QuestOnlyBackend
    from qwenquest.memory import ReqToTokenPool
    from tests.workloads import fill_rows_normal_, torch_generator

    max_ctx = ((prefix + total_steps + 1 + PAGE - 1) // PAGE) * PAGE
    rows = n_req * max_ctx + 1
    # the engine's max_context_len (req_to_token and Quest storage); pool rows stay max_ctx per request
    limit = max_ctx if context_limit is None else max(max_ctx, context_limit)
    gen = torch_generator(dev, seed)
    k_phys, v_phys = [], []
    for r in range(resident):
        scale = torch.exp(0.5 * torch.randn(KV, D, generator=gen, device=dev))
        kb = torch.empty((rows, KV, D), dtype=torch.bfloat16, device=dev)
        vb = torch.empty((rows, KV, D), dtype=torch.bfloat16, device=dev)
        fill_rows_normal_(kb, scale, gen)
        fill_rows_normal_(vb, scale, gen)
        k_phys.append(kb)
        v_phys.append(vb)
    pool = _Pool(k_phys, v_phys, layers)
    r2t = ReqToTokenPool(n_req, limit, dev)
    # request i, position p -> row 1 + i * max_ctx + p (future decode positions pre-mapped)
    r2t.req_to_token[:, :max_ctx].copy_(
        (1 + torch.arange(n_req, device=dev)[:, None] * max_ctx + torch.arange(max_ctx, device=dev)[None])
        .to(torch.int32))
    backend = B200QuestOnlyBackend(r2t, pool, {"algorithm": "quest", "top_k": TOP_K, "quest_page_size": PAGE})
    q = backend.quest
    # prefill bounds of every request for the resident buffers, copied to their aliases
    for r in range(min(resident, layers)):
        for i in range(n_req):
            q.update_prefill_representations(r, i, k_phys[r], r2t.req_to_token[i, :prefix])
    for layer in range(resident, layers):
        q.page_k_bounds[layer].copy_(q.page_k_bounds[layer % resident])
        q.running_k_min[layer].copy_(q.running_k_min[layer % resident])
        q.running_k_max[layer].copy_(q.running_k_max[layer % resident])
    q.running_token_count.fill_(prefix % PAGE)
    q.running_page_idx.fill_(prefix // PAGE)
    backend._skip_first_decode_update.fill_(1)  # prefill covered the last prompt token
    # per-layer decode inputs
    qs = torch.randn((layers, n_req, H, D), generator=gen, device=dev).to(torch.bfloat16)
    ks = torch.randn((layers, n_req, KV, D), generator=gen, device=dev).to(torch.bfloat16)
    vs = torch.randn((layers, n_req, KV, D), generator=gen, device=dev).to(torch.bfloat16)
    torch.cuda.synchronize(dev)
    return backend, pool, r2t, max_ctx, (qs, ks, vs)


def make_batches(dev, backend, pool, r2t, max_ctx, total_steps, n_req=N_REQ, prefix=PREFIX):
    from types import SimpleNamespace

    from qwenquest.batch import ForwardBatch, ForwardMode

    reqs = torch.arange(n_req, dtype=torch.int64, device=dev)
    batches = []
    for s in range(total_steps):
        pos = torch.full((n_req,), prefix + s, dtype=torch.int64, device=dev)
        out_loc = 1 + reqs * max_ctx + pos
        batches.append(ForwardBatch(
            forward_mode=ForwardMode.DECODE, input_ids=torch.zeros(n_req, dtype=torch.int64, device=dev),
            positions=pos, req_pool_indices=reqs, seq_lens=pos + 1, out_cache_loc=out_loc,
            req_to_token_pool=r2t, token_to_kv_pool=pool, attn_backend=backend))
    layers = [SimpleNamespace(layer_id=i, scaling=D ** -0.5, num_heads=H, num_kv_heads=KV, head_dim=D)
              for i in range(pool.num_layers)]
    return batches, layers


def run_step(backend, batch, layers, qkv):
    qs, ks, vs = qkv
    backend.init_forward_metadata(batch)
    out = None
    for layer in layers:
        li = layer.layer_id
        out = backend.forward(qs[li], ks[li], vs[li], layer, batch)
    return out


# --------------------------------------------------------------------------- prefill case


def prefill_case(args) -> None:
    """``--case prefill``: the K/V write + Quest bounds of one 32 768-token prefill, 48 layers.

    Fused: one ``qq_quest_extend_kv`` launch per layer (new K/V rows into the
    pool and the layer's bounds from the same registers).  Reference order:
    ``set_kv_buffer`` per layer (two index_put launches), then the bounds of
    all 48 layers from the pool after the last layer (one
    ``qq_quest_bounds_prefill`` launch, the reference's
    ``_update_quest_for_extend`` as one kernel).  The dense prefill attention
    is the same in both and not timed.  Four distinct K/V inputs (64 MB each)
    rotate over the layers, so each launch reads beyond L2.
    """
    from qwenquest_b200.backends import B200QuestOnlyBackend
    from qwenquest.batch import ForwardBatch, ForwardMode
    from qwenquest.memory import ReqToTokenPool

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    T, n_layers, nin = PREFIX, args.layers, 4
    gen = torch.Generator(device=dev).manual_seed(args.seed)
    k_phys = [torch.zeros((T + 1, KV, D), dtype=torch.bfloat16, device=dev) for _ in range(RESIDENT)]
    v_phys = [torch.zeros((T + 1, KV, D), dtype=torch.bfloat16, device=dev) for _ in range(RESIDENT)]
    pool = _Pool(k_phys, v_phys, n_layers)
    max_ctx = T + PAGE
    r2t = ReqToTokenPool(1, max_ctx, dev)
    loc = (torch.randperm(T, generator=gen, device=dev) + 1).to(torch.int64)
    r2t.req_to_token[0, :T] = loc.to(torch.int32)
    backend = B200QuestOnlyBackend(r2t, pool, {"algorithm": "quest", "top_k": TOP_K, "quest_page_size": PAGE})
    ks = [torch.randn((T, KV, D), generator=gen, device=dev).to(torch.bfloat16) for _ in range(nin)]
    vs = [torch.randn((T, KV, D), generator=gen, device=dev).to(torch.bfloat16) for _ in range(nin)]
    batch = ForwardBatch(
        forward_mode=ForwardMode.EXTEND, input_ids=torch.zeros(T, dtype=torch.int64, device=dev),
        positions=torch.arange(T, device=dev), req_pool_indices=torch.zeros(1, dtype=torch.int64, device=dev),
        seq_lens=torch.full((1,), T, dtype=torch.int64, device=dev), out_cache_loc=loc, req_to_token_pool=r2t,
        token_to_kv_pool=pool, attn_backend=backend, extend_prefix_lens=torch.zeros(1, dtype=torch.int64, device=dev),
        extend_seq_lens=torch.full((1,), T, dtype=torch.int64, device=dev))
    plan = backend._extend_plan(batch)
    q = backend.quest
    indices = r2t.req_to_token[0, :T]
    kb = [pool.get_key_buffer(i) for i in range(n_layers)]

    def fused():
        for li in range(n_layers):
            backend._extend_write(ks[li % nin], vs[li % nin], li, plan)

    def reference_order():
        for li in range(n_layers):
            pool.set_kv_buffer(li, loc, ks[li % nin], vs[li % nin])
        q.update_prefill_representations_all_layers(0, kb, indices)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            fn()
        b.record()
        torch.cuda.synchronize(dev)
        return a.elapsed_time(b) / args.steps

    clocks = ClockSampler(0)  # sampled over both timed loops (a 48-layer step takes ~1.5 ms)
    clocks.start()
    time.sleep(0.3)
    ref_ms = timed(reference_order)
    ref_state = [t.clone() for t in (q.page_k_bounds, q.running_k_min, q.running_k_max)]
    ms = timed(fused)
    clock_info = clocks.stop()
    backend.check_errors()
    same = all(torch.equal(a, b) for a, b in zip(ref_state, (q.page_k_bounds, q.running_k_min, q.running_k_max),
                                                  strict=True))
    row = KV * D * 2
    pages = T // PAGE
    per_launch = T * row * 4 + T * 8 + pages * KV * D * 4  # K/V read + written, out_cache_loc, bounds
    launch_s = ms / 1e3 / n_layers
    achieved = per_launch / launch_s / 1e9
    peak, peak_kind = measured_peaks()
    line = {
        "case": "prefill", "metric": "prefill K/V write + Quest bounds, tokens/s", "value": T / (ms / 1e3),
        "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "dtype": "bf16", "data": "synthetic (seeded N(0,1) K/V)",
        "config": {"workload": f"one {T}-token prefill, {n_layers} layers, 4 KV heads x 128, bf16, page 64, "
                               "pool rows in a seeded random order",
                   "l2": "4 distinct 64 MB K/V inputs rotate over the layers"},
        "reference_order": {"ms_per_step": ref_ms, "value": T / (ref_ms / 1e3),
                            "launches_per_step": 2 * n_layers + 1},
        "speedup_vs_reference_order": ref_ms / ms,
        "bounds_identical": same,
        "gpu_launches": n_layers * args.steps,
        "roofline": {"bound": "hbm", "kernel": "extend_kv", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "algorithmic_bytes_per_launch": per_launch, "peak_kind": peak_kind},
        "clocks": clock_info,
    }
    print(json.dumps(line), flush=True)


def prefill_attn_case(args) -> None:
    """``--case prefill_attn``: dense causal prefill attention of one ``--prefill-tokens``-token
    request (config 4's prompt, 32 768 by default), 32 query / 4 KV heads x 128, bf16.

    B200: one ``qq_extend_attention`` launch (tcgen05, K/V rows read in place
    through ``req_to_token``).  Reference: its own ``forward_extend`` loop body
    (``attention/base.py:78-93``) on the same GPU: ``k_buf[locs]`` /
    ``v_buf[locs]`` gathers, then ``extend_attention`` (``ops.py:18-45``:
    ``repeat_interleave`` and torch SDPA with ``is_causal``).  FLOPs: 4 x H x D
    per visible (query, key) pair.  Pool rows in a seeded random order.
    """
    from qwenquest.attention.ops import extend_attention as ref_extend

    from qwenquest_b200 import _lib
    from qwenquest_b200.hisparse import host_device_pointer
    from qwenquest_b200.kernels import extend_tiles
    from qwenquest_b200.quest import stream_of

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n = args.prefill_tokens
    gen = torch.Generator(device=dev).manual_seed(args.seed)
    rows = n + 1
    k = torch.randn((rows, KV, D), generator=gen, device=dev).to(torch.bfloat16)
    v = torch.randn((rows, KV, D), generator=gen, device=dev).to(torch.bfloat16)
    qs = [torch.randn((n, H, D), generator=gen, device=dev).to(torch.bfloat16) for _ in range(2)]
    r2t = (torch.randperm(n, generator=gen, device=dev) + 1).to(torch.int32)[None].contiguous()
    scaling = D ** -0.5
    lib = _lib.load()
    i64 = dict(dtype=torch.int64, device=dev)
    arrays = [torch.zeros(1, **i64), torch.full((1,), n, **i64), torch.zeros(1, **i64), torch.zeros(1, **i64)]
    batch = _lib.QQExtendBatch(arrays[0].data_ptr(), arrays[1].data_ptr(), arrays[2].data_ptr(),
                               arrays[3].data_ptr(), 0, n, 1, n)
    table = _lib.QQTokenTable(r2t.data_ptr(), r2t.stride(0), 1)
    tiles = torch.tensor(extend_tiles([n], [0]), dtype=torch.int32, device=dev)
    out = torch.empty((n, H * D), dtype=torch.bfloat16, device=dev)
    err = torch.zeros(1, dtype=torch.int32).pin_memory()
    err_dev = host_device_pointer(err)
    stream = stream_of(dev)
    step = [0]

    def ours():
        q = qs[step[0] % 2]
        step[0] += 1
        rc = lib.qq_extend_attention(batch, table, tiles.data_ptr(), tiles.numel(), q.data_ptr(), _lib.QQ_BF16, H,
                                     KV, D, q.stride(0), k.data_ptr(), v.data_ptr(), k.stride(0), rows, scaling,
                                     out.data_ptr(), out.stride(0), err_dev, stream)
        _lib.check(rc, "extend attention")

    locs = r2t[0].long()

    def reference():
        q = qs[step[0] % 2]
        step[0] += 1
        return ref_extend(q, k[locs], v[locs], prefix_len=0, scaling=scaling)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            fn()
        b.record()
        torch.cuda.synchronize(dev)
        return a.elapsed_time(b) / args.steps

    clocks = ClockSampler(0)
    clocks.start()
    time.sleep(0.3)
    ref_ms = timed(reference)
    ms = timed(ours)
    clock_info = clocks.stop()
    torch.cuda.synchronize(dev)
    _lib.raise_device_error(int(err[0]), "(extend attention)")
    step[0] = 0
    ref_out = reference()
    step[0] = 0
    ours()
    torch.cuda.synchronize(dev)
    a_, b_ = out.float(), ref_out.float()
    step_ = torch.exp2(torch.floor(torch.log2(b_.abs().clamp_min(1e-30))) - 7)
    within = bool(((a_ - b_).abs() <= torch.clamp(step_, min=2e-2)).all())
    flops = 4.0 * H * D * n * (n + 1) / 2
    achieved = flops / (ms / 1e3) / 1e12
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        peak, peak_kind = float(peaks["bf16_tflops"]), "measured (cuBLAS bf16 burst)"
    except (OSError, KeyError, ValueError):
        peak, peak_kind = 1590.0, "fallback"
    line = {
        "case": "prefill_attn", "metric": "dense causal prefill attention, TFLOP/s (causal FLOPs)",
        "value": achieved, "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "dtype": "bf16", "data": "synthetic (seeded N(0,1))",
        "config": {"workload": f"one {n}-token prefill, 1 layer, 32 query / 4 KV heads x 128, bf16, "
                               "pool rows in a seeded random order",
                   "l2": f"Q ({n * H * D * 2 / 1e6:.0f} MB per step, two inputs alternating) larger than L2"},
        "tokens_per_s": n / (ms / 1e3),
        "reference": {"ms_per_step": ref_ms, "value": flops / (ref_ms / 1e3) / 1e12,
                      "path": "k_buf[locs], v_buf[locs], repeat_interleave, torch SDPA (is_causal)"},
        "speedup_vs_reference": ref_ms / ms,
        "within_tolerance_of_reference": within,
        "gpu_launches": args.steps,
        "roofline": {"bound": "tensor", "kernel": "prefill_attn", "achieved": achieved, "peak": peak,
                     "unit": "TFLOP/s", "frac": achieved / peak, "peak_kind": peak_kind},
        "clocks": clock_info,
    }
    print(json.dumps(line), flush=True)


def moe_case(args) -> None:
    """``--case moe``: one Qwen3-30B-A3B MoE block (hidden 2048, 128 experts of 768, top 8,
    bf16, weights N(0, 0.02)) at config 4's decode batch of one GPU (``--moe-tokens``,
    8) and a 32K-token prefill.

    B200: ``B200SparseMoeBlock`` (the reference's routing, then ``qq_moe_experts``:
    two tcgen05 grouped GEMMs and the combine).  Reference: its own
    ``Qwen3MoeSparseMoeBlock.forward`` (per-expert loop) on the same GPU.
    Decode is bound by the distinct experts' weight bytes (HBM); prefill by
    the FLOPs (6 x pairs x hidden x intermediate).
    """
    from qwenquest.config import Qwen3MoeConfig
    from qwenquest.model.qwen3_moe import Qwen3MoeSparseMoeBlock

    from qwenquest_b200.moe import B200SparseMoeBlock

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = Qwen3MoeConfig()
    with torch.device(dev):
        blk = Qwen3MoeSparseMoeBlock(cfg).to(torch.bfloat16)
    gen = torch.Generator(device=dev).manual_seed(args.seed)
    with torch.no_grad():
        for p_ in blk.parameters():
            p_.copy_(torch.randn(p_.shape, generator=gen, device=dev) * 0.02)
    ours = B200SparseMoeBlock(blk)
    hidden, inter, k = cfg.hidden_size, cfg.moe_intermediate_size, cfg.num_experts_per_tok
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        tflops_peak, hbm_peak, kind = float(peaks["bf16_tflops"]), float(peaks["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        tflops_peak, hbm_peak, kind = 1590.0, 6650.0, "fallback"

    def timed(fn, x, steps):
        for _ in range(args.warmup):
            fn(x)
        torch.cuda.synchronize(dev)
        a_, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a_.record()
        for _ in range(steps):
            fn(x)
        b_.record()
        torch.cuda.synchronize(dev)
        return a_.elapsed_time(b_) / steps

    results = {}
    clocks = ClockSampler(0)
    clocks.start()
    time.sleep(0.3)
    with torch.no_grad():
        for name, tokens in (("decode", args.moe_tokens), ("prefill", args.moe_prefill_tokens)):
            x = (torch.randn((tokens, hidden), generator=gen, device=dev)).to(torch.bfloat16)
            steps = args.steps if name == "decode" else max(2, args.steps // 10)
            ref_ms = timed(blk, x, steps)
            ms = timed(ours, x, steps)
            out, ref = ours(x), blk(x)
            ours.check_errors()
            tol = 2 * 2.0 ** -8 * float(ref.abs().max())
            within = float((out.float() - ref.float()).abs().max()) <= tol
            experts = torch.topk(torch.softmax(blk.gate(x).float(), -1), k, dim=-1).indices
            active = int(torch.unique(experts).numel())
            wbytes = active * 3 * hidden * inter * 2
            flops = 6.0 * tokens * k * hidden * inter
            results[name] = {"tokens": tokens, "ms": ms, "reference_ms": ref_ms, "speedup_vs_reference": ref_ms / ms,
                             "active_experts": active, "weight_gb_s": wbytes / (ms / 1e3) / 1e9,
                             "tflops": flops / (ms / 1e3) / 1e12, "within_tolerance_of_reference": within}
            del x
    clock_info = clocks.stop()
    dec, pre = results["decode"], results["prefill"]
    line = {
        "case": "moe", "metric": "Qwen3-MoE block, decode us per layer (8 tokens)", "value": dec["ms"] * 1e3,
        "unit": "us/layer", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dec["ms"],
        "higher_is_better": False, "dtype": "bf16", "data": "synthetic (seeded N(0, 0.02) weights, N(0,1) tokens)",
        "config": {"workload": "Qwen3-30B-A3B MoE block: hidden 2048, 128 experts x 768, top 8, bf16",
                   "decode_tokens": dec["tokens"], "prefill_tokens": pre["tokens"]},
        "decode": dec, "prefill": pre,
        "gpu_launches": 3 * args.steps,
        "roofline": {"decode": {"bound": "hbm", "achieved": dec["weight_gb_s"], "peak": hbm_peak, "unit": "GB/s",
                                "frac": dec["weight_gb_s"] / hbm_peak, "peak_kind": kind},
                     "prefill": {"bound": "tensor", "achieved": pre["tflops"], "peak": tflops_peak,
                                 "unit": "TFLOP/s", "frac": pre["tflops"] / tflops_peak, "peak_kind": kind}},
        "clocks": clock_info,
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- configs 2 and 3


def _decode_inputs(dev, gen, steps, n_layers, n_req, q_ar=0.0):
    """Per-step decode inputs ``[steps, layers, n_req, ...]`` (bf16): q (AR(1) over steps when q_ar), new K/V."""
    q = torch.empty((steps, n_layers, n_req, H, D), dtype=torch.bfloat16, device=dev)
    state = torch.randn((n_layers, n_req, H, D), generator=gen, device=dev)
    for s in range(steps):
        if s:
            state = q_ar * state + torch.randn(state.shape, generator=gen, device=dev) if q_ar else \
                torch.randn(state.shape, generator=gen, device=dev)
        q[s].copy_(state)
    k = torch.randn((steps, n_layers, n_req, KV, D), generator=gen, device=dev).to(torch.bfloat16)
    v = torch.randn((steps, n_layers, n_req, KV, D), generator=gen, device=dev).to(torch.bfloat16)
    return q, k, v


def _kernel_ms(backend, batches, layers, inputs, first, last) -> dict:
    """Mean CUDA-event duration per kernel over steps [first, last) (the backend's per-launch events)."""
    backend.kernel_events = {}
    _timed_steps(backend, batches, layers, inputs, first, last)
    kev, backend.kernel_events = backend.kernel_events, None
    return {k: statistics.mean(a.elapsed_time(b) for a, b in v) for k, v in kev.items()}


def _timed_steps(backend, batches, layers, inputs, first, last):
    qs, ks, vs = inputs
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for s in range(first, last):
        run_step(backend, batches[s], layers, (qs[s], ks[s], vs[s]))
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b)


def config2_case(args) -> None:
    """``--case config2``: 16 ragged requests (14 at 65,537-131,073 tokens, 2 dense), 48 layers, Mode 2.

    K = s * (W + N(0,1)) with W a per-(head, channel) random walk along the
    positions (step N(0, 0.02^2)) and s ~ LogNormal(0, 0.5) per channel;
    V = s * N(0,1).  ``RESIDENT`` physical KV buffers alias the 48 layers as
    in config 1.  Steps go through the drop-in backend exactly as config 1.
    """
    from types import SimpleNamespace

    from qwenquest_b200.backends import B200QuestOnlyBackend
    from qwenquest.batch import ForwardBatch, ForwardMode
    from qwenquest.memory import ReqToTokenPool
    from tests.workloads import torch_generator

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    rng = np.random.default_rng(args.seed + 2)
    prefixes = [int(x) for x in rng.integers(65536, 131073, size=14)]
    prefixes = [x + 1 if x % PAGE == 0 else x for x in prefixes] + [int(x) for x in rng.integers(1, 2048, size=2)]
    n_req, n_layers, resident = len(prefixes), args.layers, min(args.resident, args.layers)
    warm = args.warmup
    total = warm + args.steps
    kstep = min(5, args.steps)  # steps of the per-kernel timing pass, after the timed ones
    total += kstep
    max_ctx = ((max(prefixes) + total + 1 + PAGE - 1) // PAGE) * PAGE
    rows = n_req * max_ctx + 1
    gen = torch_generator(dev, args.seed + 2)
    k_phys, v_phys = [], []
    for _ in range(resident):
        k_phys.append(torch.zeros((rows, KV, D), dtype=torch.bfloat16, device=dev))
        v_phys.append(torch.zeros((rows, KV, D), dtype=torch.bfloat16, device=dev))
    pool = _Pool(k_phys, v_phys, n_layers)
    r2t = ReqToTokenPool(n_req, max_ctx, dev)
    r2t.req_to_token.copy_(
        (1 + torch.arange(n_req, device=dev)[:, None] * max_ctx + torch.arange(max_ctx, device=dev)[None])
        .to(torch.int32))
    backend = B200QuestOnlyBackend(r2t, pool, {"algorithm": "quest", "top_k": TOP_K, "quest_page_size": PAGE})
    q = backend.quest
    for r in range(resident):
        scale = torch.exp(0.5 * torch.randn(KV, D, generator=gen, device=dev))
        for i, n in enumerate(prefixes):
            walk = torch.randn((n, KV, D), generator=gen, device=dev).mul_(0.02).cumsum_(0)
            k = walk.add_(torch.randn((n, KV, D), generator=gen, device=dev)).mul_(scale)
            base = 1 + i * max_ctx
            k_phys[r][base:base + n].copy_(k)
            v_phys[r][base:base + n].copy_(torch.randn((n, KV, D), generator=gen, device=dev).mul_(scale))
            del walk, k
            q.update_prefill_representations(r, i, k_phys[r], r2t.req_to_token[i, :n])
    for layer in range(resident, n_layers):
        q.page_k_bounds[layer].copy_(q.page_k_bounds[layer % resident])
        q.running_k_min[layer].copy_(q.running_k_min[layer % resident])
        q.running_k_max[layer].copy_(q.running_k_max[layer % resident])
    pre = torch.tensor(prefixes, dtype=torch.int64, device=dev)
    q.running_token_count.copy_((pre % PAGE).to(torch.int32))
    q.running_page_idx.copy_((pre // PAGE).to(torch.int32))
    backend._skip_first_decode_update.fill_(1)
    inputs = _decode_inputs(dev, gen, total, n_layers, n_req)
    reqs = torch.arange(n_req, dtype=torch.int64, device=dev)
    batches = []
    for s in range(total):
        pos = pre + s
        batches.append(ForwardBatch(
            forward_mode=ForwardMode.DECODE, input_ids=torch.zeros(n_req, dtype=torch.int64, device=dev),
            positions=pos, req_pool_indices=reqs, seq_lens=pos + 1, out_cache_loc=1 + reqs * max_ctx + pos,
            req_to_token_pool=r2t, token_to_kv_pool=pool, attn_backend=backend))
    layers = [SimpleNamespace(layer_id=i, scaling=D ** -0.5, num_heads=H, num_kv_heads=KV, head_dim=D)
              for i in range(n_layers)]
    torch.cuda.synchronize(dev)
    _timed_steps(backend, batches, layers, inputs, 0, warm)
    clocks = ClockSampler(0)
    clocks.start()
    ms = _timed_steps(backend, batches, layers, inputs, warm, warm + args.steps)
    clock_info = clocks.stop()
    kernel_ms = _kernel_ms(backend, batches, layers, inputs, warm + args.steps, total)
    backend.check_errors()
    # algorithmic bytes per layer-step at the timed steps' mean length
    step_bytes = 0
    for n in prefixes:
        L = n + 1 + warm + args.steps // 2
        step_bytes += 4_233_216 + 2048 * (L // PAGE) if L > TOP_K else 30_720 + 2052 * L
    value = n_layers * args.steps / (ms / 1e3)
    peak, peak_kind = measured_peaks()
    gbs = step_bytes * value / 1e9
    print(json.dumps({
        "case": "config2", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": 1, "steps": args.steps,
        "warmup": warm, "ms_per_step": ms / args.steps, "higher_is_better": True, "dtype": "bf16",
        "data": "synthetic (K = s*(random walk, step N(0,0.02^2), + N(0,1)), V = s*N(0,1), q N(0,1))",
        "config": {"workload": "config2: 16 requests (14 long at 65,537-131,073 tokens ending in a partial page, "
                               "2 dense-fallback), 48 layers, Quest top_k 2048 / page 64, quest mode",
                   "prefixes": prefixes, "resident_kv_layers": resident,
                   "l2": "inputs larger than L2 (~109 MB of distinct data per layer-step)"},
        "layer_step_bytes": step_bytes, "layer_step_gbs": gbs,
        "kernel_ms": kernel_ms,
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                     "peak_kind": peak_kind, "scope": "whole layer step"},
        "clocks": clock_info,
    }), flush=True)


def config3_case(args) -> None:
    """``--case config3``: Mode 3 (HiSparse), 32 requests at 65,536 tokens, 48 layers.

    The full KV lives in the pinned host tier (``host_layers=1``: the 48
    layers share one host buffer, as the full 48-layer history would need
    ~200 GB of host RAM; the bytes moved are the same), each request keeps a
    4096 + 1 slot hot buffer per layer, and decode queries follow
    q[t+1] = 0.9 q[t] + N(0,1), so each step misses part of its selection.
    Prefill is admitted through ``on_extend_finished`` (host backup, hot
    buffer, bounds).  Reported: layer-steps/s after warm-up, the hit rate and
    the swap-in bytes of the timed steps, against the host-link roofline
    (pinned host -> device copy bandwidth measured in the same run).
    """
    from types import SimpleNamespace

    from qwenquest_b200.backends import B200QuestHiSparseBackend
    from qwenquest.batch import ForwardBatch, ForwardMode
    from qwenquest.memory import MHATokenToKVPool, ReqToTokenPool
    from tests.workloads import fill_rows_normal_, torch_generator

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n_req, prefix, n_layers, buf = 32, 65536, args.layers, 4096
    warm = max(args.warmup, 8)
    kstep = min(5, args.steps)
    total = warm + args.steps + kstep
    # (one extra page: the eager backup takes one host row per request and step)
    max_ctx = ((prefix + total + 1 + PAGE - 1) // PAGE) * PAGE + PAGE
    gen = torch_generator(dev, args.seed + 3)
    r2t = ReqToTokenPool(n_req, max_ctx, dev)
    pool = MHATokenToKVPool(prefix, n_layers, KV, D, torch.bfloat16, dev)
    backend = B200QuestHiSparseBackend(
        r2t, pool, {"algorithm": "quest", "top_k": TOP_K, "quest_page_size": PAGE, "device_buffer_size": buf},
        host_pool_size=n_req * max_ctx, host_layers=1)
    scale = torch.exp(0.5 * torch.randn(KV, D, generator=gen, device=dev))
    locs = torch.arange(1, prefix + 1, dtype=torch.int64, device=dev)
    for _ in range(n_req):
        slot = r2t.alloc()
        r2t.req_to_token[slot, :prefix] = locs.to(torch.int32)
        for li in range(n_layers):
            fill_rows_normal_(pool.k_buffer[li][1:], scale, gen)
            fill_rows_normal_(pool.v_buffer[li][1:], scale, gen)
        one = torch.ones(1, dtype=torch.int64, device=dev)
        backend.on_extend_finished(ForwardBatch(
            forward_mode=ForwardMode.EXTEND, input_ids=torch.zeros(prefix, dtype=torch.int64, device=dev),
            positions=locs - 1, req_pool_indices=one * slot, seq_lens=one * prefix, out_cache_loc=locs,
            req_to_token_pool=r2t, token_to_kv_pool=pool, attn_backend=backend,
            extend_prefix_lens=one * 0, extend_seq_lens=one * prefix))
        r2t.req_to_token[slot, :prefix] = 0  # the engine frees the prefill rows after admission
    torch.cuda.synchronize(dev)
    inputs = _decode_inputs(dev, gen, total, n_layers, n_req, q_ar=0.9)
    reqs = torch.arange(n_req, dtype=torch.int64, device=dev)
    batches = []
    for s in range(total):
        pos = torch.full((n_req,), prefix + s, dtype=torch.int64, device=dev)
        batches.append(ForwardBatch(
            forward_mode=ForwardMode.DECODE, input_ids=torch.zeros(n_req, dtype=torch.int64, device=dev),
            positions=pos, req_pool_indices=reqs, seq_lens=pos + 1, out_cache_loc=None,
            req_to_token_pool=r2t, token_to_kv_pool=pool, attn_backend=backend))
    layers = [SimpleNamespace(layer_id=i, scaling=D ** -0.5, num_heads=H, num_kv_heads=KV, head_dim=D)
              for i in range(n_layers)]
    stats = backend.coord.stats
    _timed_steps(backend, batches, layers, inputs, 0, warm)
    h0, m0 = stats.hits, stats.misses
    clocks = ClockSampler(0)
    clocks.start()
    ms = _timed_steps(backend, batches, layers, inputs, warm, warm + args.steps)
    clock_info = clocks.stop()
    backend.check_errors()
    hits, misses = stats.hits - h0, stats.misses - m0
    kernel_ms = _kernel_ms(backend, batches, layers, inputs, warm + args.steps, total)
    # the host link: a 1 GiB pinned host -> device copy, best of 3
    host = torch.empty(1 << 30, dtype=torch.uint8).pin_memory()
    devbuf = torch.empty(1 << 30, dtype=torch.uint8, device=dev)
    best = float("inf")
    for _ in range(3):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        devbuf.copy_(host, non_blocking=True)
        b.record()
        torch.cuda.synchronize(dev)
        best = min(best, a.elapsed_time(b))
    link_gbs = (1 << 30) / (best / 1e3) / 1e9
    del host, devbuf
    layer_steps = n_layers * args.steps
    value = layer_steps / (ms / 1e3)
    row2 = 2 * KV * D * 2  # K and V row of one position
    swap_bytes = misses * row2 / layer_steps  # per layer-step
    L = prefix + 1 + warm + args.steps // 2
    hbm_bytes = n_req * (4_233_216 + 2048 * (L // PAGE) + 4 * buf * 4) + swap_bytes
    peak, peak_kind = measured_peaks()
    t_hbm = hbm_bytes / (peak * 1e9)
    t_link = swap_bytes / (link_gbs * 1e9)
    t_roof = max(t_hbm, t_link)
    print(json.dumps({
        "case": "config3", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": 1, "steps": args.steps,
        "warmup": warm, "ms_per_step": ms / args.steps, "higher_is_better": True, "dtype": "bf16",
        "data": "synthetic (K, V = s*N(0,1); q AR(1), rho 0.9)",
        "config": {"workload": "config3: 32 requests x 65,536 tokens, 48 layers, HiSparse (pinned host tier, "
                               "4096+1 slot hot buffer), Quest top_k 2048 / page 64", "host_layers": 1},
        "hit_rate": hits / max(1, hits + misses), "misses_per_layer_step": misses / layer_steps,
        "swap_in_bytes_per_layer_step": swap_bytes, "hbm_bytes_per_layer_step": hbm_bytes,
        "kernel_ms": kernel_ms,
        "host_link": {"achieved_gbs": swap_bytes * value / 1e9, "pinned_h2d_copy_gbs": link_gbs},
        "roofline": {"bound": "host link" if t_link >= t_hbm else "hbm",
                     "roofline_layer_steps_per_s": 1.0 / t_roof, "frac": value * t_roof,
                     "hbm_peak_gbs": peak, "peak_kind": peak_kind},
        "clocks": clock_info,
    }), flush=True)


# --------------------------------------------------------------------------- config 0


def config0_case(args) -> None:
    """``--case config0``: one request with an 8 192-token prefix (L = 8193, 128 candidate pages), one layer.

    4,495,360 algorithmic bytes per layer-step (under a microsecond at HBM
    speed): latency-bound, so the line reports microseconds per layer-step
    (lower is better) for the captured step (``DecodeStepGraph``: the step's
    bounds fold + the fused selection / attention call), the eager calls, and
    per kernel.  K, V = N(0,1) x LogNormal(0,0.5) per channel, q N(0,1); the
    benchmark's four planted pages move only the selection, not the work.
    """
    from qwenquest_b200.graphs import DecodeStepGraph

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    prefix, steps, warm = 8192, max(args.steps, 100), args.warmup
    total = 2 * (warm + steps) + warm + 5 + 2
    backend, pool, r2t, max_ctx, qkv = build_config1(dev, total, args.seed, n_req=1, prefix=prefix, layers=1,
                                                     resident=1)
    batches, layers = make_batches(dev, backend, pool, r2t, max_ctx, total, n_req=1, prefix=prefix)
    qs, ks, vs = qkv
    cur = [0]

    def take(n):
        cur[0] += n
        return range(cur[0] - n, cur[0])

    def timed(run, rng):
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for st in rng:
            run(st)
        b.record()
        torch.cuda.synchronize(dev)
        return a.elapsed_time(b) * 1e3 / len(rng)  # us per step

    eager = lambda st: run_step(backend, batches[st], layers, qkv)  # noqa: E731
    for st in take(warm):
        eager(st)
    eager_us = timed(eager, take(steps))
    graph = DecodeStepGraph(backend, layers, batches[cur[0]], qs, ks, vs)
    replay = lambda st: graph.replay(batches[st])  # noqa: E731
    for st in take(warm):
        replay(st)
    clocks = ClockSampler(0)
    clocks.start()
    graph_us = timed(replay, take(steps))
    clock_info = clocks.stop()
    kernel_ms = _kernel_ms(backend, batches, layers, qkv_steps(qkv, total), *_span(take(5)))
    backend.check_errors()
    step_bytes = 4_233_216 + 2048 * (prefix // PAGE)
    print(json.dumps({
        "case": "config0", "metric": "Quest sparse-decode latency per layer-step (1 request)", "value": graph_us,
        "unit": "us", "n_gpus": 1, "steps": steps, "warmup": warm, "ms_per_step": graph_us / 1e3,
        "higher_is_better": False, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) x LogNormal(0,0.5) per-channel K/V, N(0,1) q)",
        "config": {"workload": "config0: 1 request x 8192-token prefix (L = 8193, 128 candidate pages), 1 layer, "
                               "Quest top_k 2048 / page 64, Qwen3-30B-A3B attention (32q/4kv x 128, bf16)",
                   "layer_step_bytes": step_bytes,
                   "l2": "one request: ~4.5 MB per layer-step stays in L2 between steps (latency case)"},
        "paths": {"graph_us": graph_us, "eager_us": eager_us,
                  "what": "per layer-step: the step's bounds fold + one fused selection / attention call"},
        "kernel_us": {k: v * 1e3 for k, v in kernel_ms.items()},
        "layer_step_gbs": step_bytes / (graph_us * 1e-6) / 1e9,
        "clocks": clock_info,
    }), flush=True)


# --------------------------------------------------------------------------- config 4


def config4_case(args) -> None:
    """``--case config4``: end-to-end decode through the reference ``Engine`` on one GPU's shard.

    The benchmark's config 4 is a random-init Qwen3-30B-A3B (48 layers, hidden 2048,
    32 / 4 heads x 128, 128 experts top-8, moe_intermediate 768, vocab 151936,
    bf16, weights ~N(0, 0.02)), batch 64 at context 32768, 128 new tokens,
    quest mode, requests sharded over 8 GPUs with only the attention backend
    replaced.  Requests are independent, so one GPU's shard (64 / 8 = 8
    requests) runs here alone: the reference's model and engine (its
    prefill, batched decode and MoE loop) with ``B200QuestOnlyBackend`` behind
    ``Engine._make_backend``, the whole integration a user makes.
    Prompts are seeded uniform-random token ids.  Reported: decode tokens/s of
    the shard (host-timed around ``Engine._decode``, synchronized), the box's
    tokens/s as 8 such shards (no collective on the path), prefill seconds,
    and the attention backend's share of the decode time (CUDA events around
    every ``forward_decode``).  The weights are drawn on the GPU with a
    seeded generator (the reference's ``init_random_weights`` draws 30.5 B
    values on the host; same distribution).
    """
    from qwenquest import Engine, EngineConfig, Qwen3MoeForCausalLM
    from qwenquest.config import Qwen3MoeConfig, parse_hisparse_config

    from qwenquest_b200 import B200QuestOnlyBackend

    class B200Engine(Engine):
        def _make_backend(self):
            sparse = parse_hisparse_config({"algorithm": "quest", "top_k": TOP_K, "quest_page_size": PAGE})
            return B200QuestOnlyBackend(self.req_to_token_pool, self.token_to_kv_pool, sparse)

    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    n_req, ctx, new = args.c4_requests, args.c4_context, args.c4_new_tokens
    t0 = time.perf_counter()
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device(dev):
            model = Qwen3MoeForCausalLM(Qwen3MoeConfig())
    finally:
        torch.set_default_dtype(prev)
    gen = torch.Generator(device=dev).manual_seed(args.seed)
    with torch.no_grad():
        for name, param in model.named_parameters():
            if name.endswith("norm.weight"):
                param.fill_(1.0)
            else:
                param.normal_(0.0, 0.02, generator=gen)
    model.eval()
    n_params = sum(p.numel() for p in model.parameters())
    moe_blocks = 0
    if args.c4_moe:
        from qwenquest_b200.moe import install_moe

        moe_blocks = install_moe(model)
    engine = B200Engine(model, EngineConfig(attention_mode="quest", max_running_requests=n_req,
                                            max_context_len=ctx + new + 1))
    init_s = time.perf_counter() - t0
    g = torch.Generator().manual_seed(args.seed + 1 + 1000 * rank)  # each rank its own shard of prompts
    prompts = [torch.randint(0, model.config.vocab_size, (ctx,), generator=g).tolist() for _ in range(n_req)]

    phase = {"prefill": 0.0, "decode": 0.0, "decode_steps": 0}
    orig_prefill, orig_decode = engine._prefill, engine._decode

    def timed_phase(fn, key):
        def run(*a, **k):
            torch.cuda.synchronize(dev)
            t = time.perf_counter()
            out = fn(*a, **k)
            torch.cuda.synchronize(dev)
            phase[key] += time.perf_counter() - t
            if key == "decode":
                phase["decode_steps"] += 1
            return out
        return run

    engine._prefill = timed_phase(orig_prefill, "prefill")
    engine._decode = timed_phase(orig_decode, "decode")
    backend = engine.attn_backend
    orig_fd = backend.forward_decode
    events = []

    def fd(q, k, v, layer, batch):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        out = orig_fd(q, k, v, layer, batch)
        e1.record()
        events.append((e0, e1))
        return out

    backend.forward_decode = fd
    outs = engine.generate(prompts, max_new_tokens=new, stop_token_ids=[])
    torch.cuda.synchronize(dev)
    backend.check_errors()
    attn_s = sum(a.elapsed_time(b) for a, b in events) / 1e3
    tokens = sum(len(o.output_ids) for o in outs)
    decode_tokens = tokens - n_req  # the first token of each request comes from its prefill
    dec_tps = decode_tokens / phase["decode"]
    box = None
    if world > 1:
        # the box: every rank decoded its own shard; tokens summed, time of the slowest rank
        from qwenquest_b200.sharding import box_totals

        (dec_max, pre_max), (n_tok,) = box_totals([phase["decode"], phase["prefill"]], [decode_tokens], dev)
        box = {"ranks": world, "decode_tokens": n_tok, "decode_s_max": dec_max, "prefill_s_max": pre_max,
               "decode_tokens_per_s": n_tok / dec_max}
        if rank != 0:
            return
    replaced = "the attention backend and the MoE blocks" if moe_blocks else "the attention backend only"
    print(json.dumps({
        "case": "config4", "metric": "end-to-end decode tokens/s (reference Engine, B200 attention backend)",
        "replaced": replaced, "moe_blocks_replaced": moe_blocks,
        "value": box["decode_tokens_per_s"] if box else dec_tps, "unit": "tokens/s", "higher_is_better": True,
        "dtype": "bf16", "shard_tokens_per_s": dec_tps,
        "data": "synthetic (random-init weights N(0, 0.02) drawn on the GPU, seeded uniform-random prompt ids)",
        "config": {"workload": f"config4 shard: {n_req} requests x {ctx}-token prompts, {new} new tokens, "
                               "random-init Qwen3-30B-A3B (48 layers, 128 experts top-8), quest mode "
                               "(top_k 2048 / page 64), the reference Engine with B200QuestOnlyBackend",
                   "params": n_params, "shard_of": 64},
        "box_tokens_per_s_8_shards": 8 * dec_tps,
        "box": box,
        "n_gpus": world,
        "decode_s": phase["decode"], "decode_steps": phase["decode_steps"], "prefill_s": phase["prefill"],
        "prefill_tokens_per_s": n_req * ctx / phase["prefill"],
        "attention_decode_s": attn_s, "attention_share_of_decode": attn_s / phase["decode"],
        "init_s": init_s, "peak_mem_gb": torch.cuda.max_memory_allocated(dev) / 1e9,
    }), flush=True)


def qkv_steps(qkv, total):
    """The same per-layer inputs for every step ([steps, layers, ...] views)."""
    return tuple(t.unsqueeze(0).expand(total, *t.shape) for t in qkv)


def _span(rng):
    return rng.start, rng.stop


# --------------------------------------------------------------------------- CPU baseline


def _cpu_sample(sample_reqs: int, min_seconds: float, seed: int, samples: int = 1) -> list[tuple[int, float]]:
    """One worker: the numpy oracle on ``sample_reqs`` requests x one layer of config 1;
    ``samples`` consecutive timings of >= ``min_seconds`` each, as (repetitions, seconds)."""
    from threadpoolctl import threadpool_limits

    from oracle.attention import decode_attention
    from oracle.bf16 import round_bf16
    from oracle.quest import OracleQuest

    threadpool_limits(1)  # one core per worker process
    rng = np.random.default_rng(seed)
    n = PREFIX + 1
    scale = rng.lognormal(0, 0.5, size=(1, KV, D)).astype(np.float32)
    ks = [round_bf16(rng.standard_normal((n, KV, D), dtype=np.float32) * scale) for _ in range(sample_reqs)]
    vs = [round_bf16(rng.standard_normal((n, KV, D), dtype=np.float32) * scale) for _ in range(sample_reqs)]
    q = round_bf16(rng.standard_normal((sample_reqs, H, D), dtype=np.float32))
    oq = OracleQuest(TOP_K, PAGE)
    oq.init_storage(0, 1, sample_reqs, n + PAGE, KV, D)
    for i in range(sample_reqs):
        oq.update_prefill_representations(0, i, ks[i], np.arange(PREFIX))
    reqs = np.arange(sample_reqs)
    seq = np.full(sample_reqs, n)
    out = []
    for _ in range(samples):
        reps, t0 = 0, time.perf_counter()
        while True:
            # the per-step bounds fold of the previous token; counters reset so repetitions stay in range
            oq.running_token_count[:] = 0
            oq.running_page_idx[:] = PREFIX // PAGE
            oq.update_decode_representations(0, reqs, np.stack([k[n - 2] for k in ks]), np.arange(sample_reqs))
            oq.maybe_finalize_decode_representations(reqs)
            oq.prepare_step(seq)
            pos, actual = oq.retrieve_topk(q, 0, reqs, query_is_bf16=True)
            for i in range(sample_reqs):
                r = pos[i, : actual[i]].astype(np.int64)
                decode_attention(q[i], ks[i][r], vs[i][r], D ** -0.5, out_bf16=True)
            reps += 1
            el = time.perf_counter() - t0
            if el >= min_seconds:
                break
        out.append((reps, el))
    return out


def reference_sample(n_req: int, steps: int, warmup: int, seed: int = 0) -> dict:
    """The reference's own ``QuestOnlyBackend`` (``src/qwenquest/attention/quest_only.py``) on CPU pools,
    timed on the host cores: ``n_req`` requests of config 1 (32 768-token prefixes, bounds built by its
    own ``update_prefill_representations``), one layer; a step is ``init_forward_metadata`` +
    ``forward`` for that layer, i.e. ``n_req / 64`` of a layer-step."""
    from types import SimpleNamespace

    from qwenquest.attention import QuestOnlyBackend
    from qwenquest.batch import ForwardBatch, ForwardMode
    from qwenquest.memory import MHATokenToKVPool, ReqToTokenPool

    threads = host_cores()
    torch.set_num_threads(threads)
    total = warmup + steps
    max_ctx = ((PREFIX + total + 1 + PAGE - 1) // PAGE) * PAGE
    gen = torch.Generator().manual_seed(seed)
    t0 = time.perf_counter()
    pool = MHATokenToKVPool(n_req * max_ctx, 1, KV, D, torch.bfloat16, "cpu")
    scale = torch.exp(0.5 * torch.randn(KV, D, generator=gen))
    for buf in (pool.k_buffer[0], pool.v_buffer[0]):
        for r0 in range(1, buf.shape[0], 1 << 16):  # N(0,1) x per-channel scale, in chunks
            r1 = min(buf.shape[0], r0 + (1 << 16))
            buf[r0:r1] = torch.randn((r1 - r0, KV, D), generator=gen).mul_(scale)
    r2t = ReqToTokenPool(n_req, max_ctx, "cpu")
    r2t.req_to_token.copy_((1 + torch.arange(n_req)[:, None] * max_ctx + torch.arange(max_ctx)[None]).to(torch.int32))
    backend = QuestOnlyBackend(r2t, pool, {"algorithm": "quest", "top_k": TOP_K, "quest_page_size": PAGE})
    for i in range(n_req):  # what the reference's _update_quest_for_extend does after a prefill
        backend.quest.update_prefill_representations(0, i, pool.k_buffer[0], r2t.req_to_token[i, :PREFIX])
        backend._skip_first_decode_update[i] = True
    layer = SimpleNamespace(layer_id=0, scaling=D ** -0.5, num_heads=H, num_kv_heads=KV, head_dim=D)
    reqs = torch.arange(n_req, dtype=torch.int64)
    setup_s = time.perf_counter() - t0
    times = []
    for s in range(total):
        pos = torch.full((n_req,), PREFIX + s, dtype=torch.int64)
        batch = ForwardBatch(forward_mode=ForwardMode.DECODE, input_ids=torch.zeros(n_req, dtype=torch.int64),
                             positions=pos, req_pool_indices=reqs, seq_lens=pos + 1,
                             out_cache_loc=1 + reqs * max_ctx + pos, req_to_token_pool=r2t, token_to_kv_pool=pool,
                             attn_backend=backend)
        q = torch.randn((n_req, H, D), generator=gen).to(torch.bfloat16)
        k = torch.randn((n_req, KV, D), generator=gen).mul_(scale).to(torch.bfloat16)
        v = torch.randn((n_req, KV, D), generator=gen).mul_(scale).to(torch.bfloat16)
        a = time.perf_counter()
        backend.init_forward_metadata(batch)
        backend.forward(q, k, v, layer, batch)
        times.append(time.perf_counter() - a)
    timed = times[warmup:]
    sec = statistics.mean(timed)
    return {
        "value": (n_req / N_REQ) / sec,
        "unit": UNIT,
        "cores": threads,
        "kind": "reference",
        "sample": f"the reference's own QuestOnlyBackend (torch {torch.__version__}, CPU, {threads} threads) on "
                  f"{n_req} of config 1's 64 requests x 1 layer, {steps} timed steps after {warmup} warm-up "
                  f"(init_forward_metadata + forward), scaled to the 64-request layer-step",
        "ms_per_layer_step": 1e3 * sec * N_REQ / n_req,
        "setup_s": setup_s,
    }


def host_cores() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


def cpu_baseline(min_seconds: float = 10.0, seed: int = 0, samples: int = 1, sample_reqs: int = 1) -> list[dict]:
    """The numpy oracle (the reference's algorithm) on all host cores: one single-threaded
    worker process per core (spawned), each timing ``samples`` consecutive bounded samples of
    config 1 (``sample_reqs`` requests x one layer, >= ``min_seconds`` each); a sample's
    throughput is the sum over the workers, scaled to the 64-request layer-step."""
    import multiprocessing as mproc

    workers = host_cores()
    with mproc.get_context("spawn").Pool(workers) as pool:
        res = pool.starmap(_cpu_sample, [(sample_reqs, min_seconds, seed + w, samples) for w in range(workers)])
    lines = []
    for k in range(samples):
        req_layers_per_s = sum(r[k][0] * sample_reqs / r[k][1] for r in res)
        reps = sum(r[k][0] for r in res)
        lines.append({
            "value": req_layers_per_s / N_REQ,
            "unit": UNIT,
            "cores": workers,
            "kind": "port",
            "sample": f"{workers} single-threaded worker processes x {sample_reqs} request x 1 layer of "
                      f"config 1, {reps} repetitions in >= {min_seconds:.1f} s (numpy oracle), scaled to "
                      f"the 64-request layer-step",
            "ms_per_request_layer": 1e3 * workers / req_layers_per_s,
        })
    return lines


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# --------------------------------------------------------------------------- main


def load_profile_traffic() -> float | None:
    p = ROOT / "profiles" / "traffic.json"
    try:
        d = json.loads(p.read_text())
        return float(d["sparse_decode_attention"]["dram_bytes_per_launch"])
    except (OSError, KeyError, ValueError, TypeError):
        return None


def measured_peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--cpu-requests", type=int, default=N_REQ,
                    help="requests of the reference's CPU sample (a layer-step of config 1 has 64)")
    ap.add_argument("--requests", type=int, default=N_REQ, help="requests per GPU (profiling cases only)")
    ap.add_argument("--layers", type=int, default=LAYERS, help="layers (profiling cases only)")
    ap.add_argument("--resident", type=int, default=RESIDENT, help="physical KV buffers")
    ap.add_argument("--context-limit", type=int, default=None,
                    help="engine max_context_len above the requests' lengths (profiling cases only)")
    ap.add_argument("--case", choices=["decode", "prefill", "prefill_attn", "moe", "config0", "config2", "config3",
                                       "config4"],
                    default="decode",
                    help="decode: the benchmark, config 1 (default); prefill: the prefill K/V write + bounds; "
                         "config2 / config3: the ragged and HiSparse benchmark configs (1 GPU each); "
                         "config4: end-to-end decode through the reference Engine, one GPU's shard; "
                         "prefill_attn: the dense causal prefill attention against the reference's")
    ap.add_argument("--prefill-tokens", type=int, default=PREFIX, help="prefill_attn: tokens of the request")
    ap.add_argument("--moe-tokens", type=int, default=8, help="moe: tokens of the decode batch (64 / 8 GPUs)")
    ap.add_argument("--moe-prefill-tokens", type=int, default=PREFIX, help="moe: tokens of the prefill batch")
    ap.add_argument("--c4-requests", type=int, default=8, help="config4: requests of the shard (64 / 8 GPUs)")
    ap.add_argument("--c4-context", type=int, default=32768, help="config4: prompt tokens per request")
    ap.add_argument("--c4-new-tokens", type=int, default=128, help="config4: tokens generated per request")
    ap.add_argument("--c4-moe", action="store_true",
                    help="config4: also replace the model's MoE blocks by B200SparseMoeBlock (the benchmark's "
                         "config replaces the attention backend only)")
    ap.add_argument("--path", choices=["graph", "eager"], default="graph",
                    help="headline path: the decode step replayed as a CUDA graph (default) or the eager calls")
    ap.add_argument("--weak", action="store_true",
                    help="--requests per GPU (weak scaling) instead of sharding --requests over the GPUs")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.case == "config4" and int(os.environ.get("WORLD_SIZE", "1")) > 1:
        # config 4 as the benchmark names it: the 64 requests sharded over the GPUs, one shard per rank
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.distributed.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=900),
                                             device_id=torch.device("cuda", local))
        try:
            config4_case(args)
        finally:
            torch.distributed.destroy_process_group()
        return
    if args.case != "decode":
        if int(os.environ.get("RANK", "0")) == 0:
            {"prefill": prefill_case, "prefill_attn": prefill_attn_case, "moe": moe_case, "config0": config0_case, "config2": config2_case,
             "config3": config3_case, "config4": config4_case}[args.case](args)
        return
    from qwenquest_b200.graphs import DecodeStepGraph
    from qwenquest_b200.sharding import max_over_ranks, shard_requests

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return
        t0 = time.perf_counter()
        cb = reference_sample(args.cpu_requests, args.steps, args.warmup, seed=args.seed)
        value = cb["value"]
        port = cpu_baseline(min_seconds=max(0.5, args.cpu_seconds / 4))[0]
        line = {
            "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * LAYERS / value,
            "higher_is_better": True, "scaling": "weak" if args.weak else "strong", "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic", "cpu_baseline": cb,
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "config": {"workload": "config1: 64 requests x 32768-token prefix, 48 layers, Quest top_k 2048 / page 64, "
                                   "Qwen3-30B-A3B attention (32q/4kv x 128, bf16), quest mode",
                       "cpu": cpu_model(), "wall_s": time.perf_counter() - t0},
            "port": {"value": port["value"], "sample": port["sample"], "cores": port["cores"],
                     "what": "the numpy restatement of the same path (oracle/), for comparison"},
        }
        print(json.dumps(line))
        return

    if world > 1:
        torch.distributed.init_process_group(
            "nccl", timeout=__import__("datetime").timedelta(seconds=120),
            device_id=torch.device("cuda", local_rank))
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    total = args.warmup + args.steps
    # five passes of W + K steps each, in this order: eager (the drop-in
    # forward calls), graph (the same steps replayed as a captured
    # DecodeStepGraph), per-kernel events (eager, two calls per layer), e2e
    # through the graph, e2e through the eager calls
    n_layers = args.layers
    # strong scaling (default): the --requests batch is sharded by request; weak: every rank decodes its own
    n_req = args.requests if args.weak else len(shard_requests([PREFIX + 1] * args.requests, rank, world))
    n_steps = 5 * total + 2
    backend, pool, r2t, max_ctx, qkv = build_config1(dev, n_steps, args.seed + 1000 * rank, n_req=n_req,
                                                     layers=n_layers, resident=min(args.resident, n_layers),
                                                     context_limit=args.context_limit)
    batches, layers = make_batches(dev, backend, pool, r2t, max_ctx, n_steps, n_req=n_req)
    qs, ks, vs = qkv
    cursor = [0]

    def take(n):
        first = cursor[0]
        cursor[0] += n
        return range(first, first + n)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)

    def timed(run, steps, clocks=None):
        """Device time of `run(s)` over `steps` (CUDA events on the compute stream, a barrier on both sides)."""
        barrier()
        if clocks is not None:
            clocks.start()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        torch.cuda.nvtx.range_push("timed")  # profilers select the timed steps by this range
        for st in steps:
            run(st)
        torch.cuda.nvtx.range_pop()
        b.record()
        barrier()
        info = clocks.stop() if clocks is not None else None
        return a.elapsed_time(b), info

    eager_step = lambda st: run_step(backend, batches[st], layers, qkv)  # noqa: E731

    # ---- eager: the drop-in calls (init_forward_metadata + forward per layer), inputs resident
    for st in take(args.warmup):
        eager_step(st)
    eager_ms, _ = timed(eager_step, take(args.steps))
    backend.check_errors()

    # ---- graph: the same steps as replays of a captured DecodeStepGraph (the headline by default)
    graph = DecodeStepGraph(backend, layers, batches[cursor[0]], qs, ks, vs)
    graph_step = lambda st: graph.replay(batches[st])  # noqa: E731
    for st in take(args.warmup):
        graph_step(st)
    clock_dev = dev.index if world == 1 else local_rank
    graph_ms, clock_info = timed(graph_step, take(args.steps), ClockSampler(clock_dev))
    backend.check_errors()
    del graph

    # ---- per-kernel durations (CUDA events on the launching stream), eager two-call path
    for st in take(args.warmup):
        eager_step(st)
    barrier()
    backend.kernel_events = {}
    for st in take(args.steps):
        eager_step(st)
    barrier()
    kev = backend.kernel_events
    backend.kernel_events = None
    kernel_ms = {k: statistics.mean(a.elapsed_time(b) for a, b in v) for k, v in kev.items()}
    launches = sum(len(v) for v in kev.values())
    backend.check_errors()

    # ---- e2e: host (pinned) inputs copied in, every layer's output copied out, each step.
    # The copies run on their own streams (a step's inputs ahead of the step,
    # into one of two buffer sets by step parity; the step's outputs behind
    # it), ordered by events, so PCIe traffic overlaps the kernels.  The timed
    # region spans every copy.
    hq, hk, hv = (t.cpu().pin_memory() for t in (qs, ks, vs))
    hout = torch.empty((n_layers, n_req, H * D), dtype=torch.bfloat16).pin_memory()
    compute = torch.cuda.current_stream(dev)
    h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def e2e_pass(bufs, step, steps):
        """`steps` with their copies: bufs[p] = (q, k, v, out) device buffers of parity p, step(st, p)
        runs step st on buffer set p; returns once every stream's work is queued."""
        step_done = [None, None]  # compute finished with the buffer set of that parity
        out_done = [None, None]  # the device->host copy finished with the output buffer of that parity
        steps = list(steps)

        def copy_inputs(i):
            p = i % 2
            if step_done[p] is not None:
                h2d.wait_event(step_done[p])
            with torch.cuda.stream(h2d):
                for dst, src in zip(bufs[p][:3], (hq, hk, hv), strict=True):
                    dst.copy_(src, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(h2d)
            return ev

        h2d.wait_stream(compute)
        d2h.wait_stream(compute)
        ready = copy_inputs(0)
        for i, st in enumerate(steps):
            p = i % 2
            compute.wait_event(ready)
            if out_done[p] is not None:
                compute.wait_event(out_done[p])
            step(st, p)
            done = torch.cuda.Event()
            done.record(compute)
            step_done[p] = done
            # the step's outputs cross PCIe (one copy) while the next step computes
            d2h.wait_event(done)
            with torch.cuda.stream(d2h):
                hout.copy_(bufs[p][3], non_blocking=True)
            out_done[p] = torch.cuda.Event()
            out_done[p].record(d2h)
            if i + 1 < len(steps):
                ready = copy_inputs(i + 1)  # the next step's inputs cross PCIe during this step
        compute.wait_stream(d2h)
        compute.wait_stream(h2d)

    def timed_e2e(bufs, step):
        e2e_pass(bufs, step, take(args.warmup))  # warm-up: the same steps, copies included
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(compute)
        t_host = time.perf_counter()
        e2e_pass(bufs, step, take(args.steps))
        host_ms = 1e3 * (time.perf_counter() - t_host) / args.steps  # enqueue time per step
        b.record(compute)
        barrier()
        return a.elapsed_time(b), host_ms

    # through two graphs (by step parity), each with its own input and stacked output buffers
    graphs = [DecodeStepGraph(backend, layers, batches[cursor[0]], qs, ks, vs, stack_outputs=True)
              for _ in range(2)]
    gbufs = [(g.q, g.k, g.v, g.out_stacked) for g in graphs]
    e2e_ms, e2e_host_ms = timed_e2e(gbufs, lambda st, p: graphs[p].replay(batches[st]))
    backend.check_errors()
    del graphs, gbufs

    # through the eager calls
    ebufs = [tuple(torch.empty_like(t) for t in (qs, ks, vs)) +
             (torch.empty((n_layers, n_req, H * D), dtype=torch.bfloat16, device=dev),) for _ in range(2)]

    def eager_e2e_step(st, p):
        dq, dk, dv, dout = ebufs[p]
        b = batches[st]
        backend.init_forward_metadata(b)
        torch.stack([backend.forward(dq[lay.layer_id], dk[lay.layer_id], dv[lay.layer_id], lay, b)
                     for lay in layers], out=dout)

    e2e_eager_ms, e2e_eager_host_ms = timed_e2e(ebufs, eager_e2e_step)
    backend.check_errors()

    graph_ms, eager_ms, e2e_ms, e2e_eager_ms = max_over_ranks([graph_ms, eager_ms, e2e_ms, e2e_eager_ms],
                                                              device=dev)  # the box is as fast as its slowest GPU
    ms, value_path = (graph_ms, "graph") if args.path == "graph" else (eager_ms, "eager")

    c = PREFIX // PAGE + 0  # candidate pages at the first timed step (F = 512 while seq_len < 32832)
    batches_per_layer_step = world if args.weak else 1  # 64-request batches the box decodes per layer step
    layer_steps = batches_per_layer_step * n_layers * args.steps
    value = layer_steps / (ms / 1e3)
    e2e_ms_head, e2e_host_head = (e2e_ms, e2e_host_ms) if value_path == "graph" else (e2e_eager_ms, e2e_eager_host_ms)
    e2e_value = layer_steps / (e2e_ms_head / 1e3)
    peak, peak_kind = measured_peaks()
    attn_ms = kernel_ms.get("sparse_decode_attention")
    achieved = n_req * ATTN_BYTES_PER_REQ / (attn_ms / 1e3) / 1e9 if attn_ms else None
    traffic = load_profile_traffic()
    step_bytes = layer_step_bytes(c, n_req)
    line = {
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms / args.steps,
        "higher_is_better": True,
        "scaling": "weak" if args.weak else "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) x LogNormal(0,0.5) per-channel K/V, N(0,1) q)",
        "config": {
            "workload": (f"config1: {args.requests} requests/GPU" if args.weak else
                         f"config1: {args.requests} requests sharded over {world} GPU(s)")
                        + " x 32768-token prefix, 48 layers, Quest top_k 2048 / page 64, "
                        "Qwen3-30B-A3B attention (32q/4kv x 128, bf16), quest mode",
            "requests_per_gpu": n_req, "layers": n_layers, "resident_kv_layers": min(args.resident, n_layers),
            "context_limit": int(r2t.max_context_len),
            "l2": f"inputs larger than L2 (each GPU's layer-step reads ~{step_bytes / 1e6:.0f} MB of distinct data)"
                  if step_bytes > 126e6 else
                  f"each GPU's layer-step reads ~{step_bytes / 1e6:.0f} MB of distinct data; the 4 resident KV "
                  f"buffers rotate over the layers, so a buffer returns after 4 layer-steps "
                  f"(~{4 * step_bytes / 1e6:.0f} MB of distinct data in between)",
            "layer_step_bytes": step_bytes,
            "layer_step_gbs": step_bytes / (ms / 1e3 / (n_layers * args.steps)) / 1e9,
            "layer_step_frac_of_peak": step_bytes / (ms / 1e3 / (n_layers * args.steps)) / 1e9 / peak,
            # the same against the nominal 8 TB/s of B200 HBM3e, and per request
            "layer_step_frac_of_nominal_8tbs": step_bytes / (ms / 1e3 / (n_layers * args.steps)) / 8e12,
            "request_layer_steps_per_s_per_gpu": n_req * (n_layers * args.steps) / (ms / 1e3),
            "kernel_ms": kernel_ms,
            "path": value_path,
            "paths": {
                "graph": {"value": layer_steps / (graph_ms / 1e3), "ms_per_step": graph_ms / args.steps,
                          "e2e": layer_steps / (e2e_ms / 1e3), "e2e_host_enqueue_ms_per_step": e2e_host_ms,
                          "what": "DecodeStepGraph.replay per step (the decode step captured once: "
                                  "fold + 48 x fused selection/attention, device-side epochs)"},
                "eager": {"value": layer_steps / (eager_ms / 1e3), "ms_per_step": eager_ms / args.steps,
                          "e2e": layer_steps / (e2e_eager_ms / 1e3),
                          "e2e_host_enqueue_ms_per_step": e2e_eager_host_ms,
                          "what": "init_forward_metadata + forward per layer (the drop-in calls Engine.generate "
                                  "makes), fused selection/attention call per layer"},
            },
        },
        "roofline": {
            "bound": "hbm",
            "kernel": "sparse_decode_attention",
            "achieved": achieved,
            "peak": peak,
            "unit": "GB/s",
            "frac": achieved / peak if achieved else None,
            "traffic": traffic,
            "algorithmic_bytes_per_launch": n_req * ATTN_BYTES_PER_REQ,
            "peak_kind": peak_kind,
        },
        "clocks": clock_info,
        "gpu_launches": launches,
        "e2e": {
            "value": e2e_value,
            "unit": UNIT,
            "h2d_bytes_per_step": int(sum(t.numel() * t.element_size() for t in (hq, hk, hv))),
            "d2h_bytes_per_step": int(hout.numel() * hout.element_size()),
            "host_enqueue_ms_per_step": e2e_host_head,
        },
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        del backend, pool, r2t, qkv, batches, hq, hk, hv, hout, ebufs
        torch.cuda.empty_cache()
        line["cpu_baseline"] = reference_sample(args.cpu_requests, 3, 2, seed=args.seed)
        line["cpu_baseline_port"] = cpu_baseline(min_seconds=args.cpu_seconds)[0]
        line["config"]["cpu"] = cpu_model()
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
