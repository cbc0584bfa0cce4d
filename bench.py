#!/usr/bin/env python
"""Prefill benchmark of the block-sparse attention path on B200.

Workload (default ``c1``): a deepseek-coder-1.3B-architecture LLaMA (24
layers, hidden 2048, 16 heads x 128, MLP 5504, vocab 32256, RoPE theta 1e5
linear x4), random-init bf16 weights, one 12288-token prompt of uniform random
ids per GPU with seeded structure spans; every layer runs the block-sparse
prefill kernel with block 64, a 4-block window, sink block, 128-token chunk
groups and the per-layer pooled top-8 blocks. A step is one full-model
prefill (logits for the last position, as generation's prefill computes).

``value`` is prompt tokens/s over all ranks (weak scaling: one prompt per
GPU, no collective on the data path). ``attn_tflops`` counts only listed
(non-masked) 64x64 blocks, 4*64*64*128 FLOP each. Other workloads:
``c2`` (8 prompts of 12288-16384 tokens split over the ranks, strong
scaling), ``c3`` (6.7B architecture, 16384 tokens), ``c0`` (the single
attention op, B=1, H=16, L=4096).

``--impl reference`` times the reference's own CPU path for the same
workload on the host cores: the dense-masked attention arithmetic of the
reference's fallback (sabrecoder_attention_triton.py:2061-2066) inside a
decoder layer, on a bounded sample (one decoder layer, scaled to the model).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "prefill tokens/s & effective sparse-attn TFLOP/s at 12K-16K ctx, 1/2/4/8 B200"

ARCH = {
    "1.3b": dict(vocab_size=32256, hidden_size=2048, intermediate_size=5504, num_hidden_layers=24,
                 num_attention_heads=16, num_key_value_heads=16),
    "6.7b": dict(vocab_size=32256, hidden_size=4096, intermediate_size=11008, num_hidden_layers=32,
                 num_attention_heads=32, num_key_value_heads=32),
    "33b": dict(vocab_size=32256, hidden_size=7168, intermediate_size=19200, num_hidden_layers=62,
                num_attention_heads=56, num_key_value_heads=8),
}
MASK = dict(block_size=64, window_size=192, num_prefix_tokens=64, num_suffix_tokens=128, max_chunk_tokens=128,
            global_last_k_chunks=0)
TOPK = 8
# The 33B workload: block 128 (4-block window), structure lists only.
MASK_C4 = dict(block_size=128, window_size=384, num_prefix_tokens=128, num_suffix_tokens=128, max_chunk_tokens=128,
               global_last_k_chunks=0)


# Fewer definitions than the 1.3B/6.7B mix: with 128-token blocks the sink, the
# 4-block window and the suffix alone are ~11 % of a 16K causal row, so this
# mix brings the structure lists to ~14 % (the config asks for ~12 %).
C4_SPAN_MIX = dict(p_class=0.01, p_function=0.04, header_frac=0.005)


def mask_text(mask, topk) -> str:
    return (f"block {mask['block_size']}, window {mask['window_size']}, sink {mask['num_prefix_tokens']}, "
            f"suffix {mask['num_suffix_tokens']}, {mask['max_chunk_tokens']}-token chunk groups"
            + (f", pooled top-{topk} per layer/head" if topk else ", structure lists only"))


def workload_text(name: str) -> str:
    """The job both arms run, independent of the rank and of the arm."""
    mask, topk = mask_cfg(name)
    arch, prompts, scaling = workload(name, 0, 1)
    if name == "c2":
        lens = [p[0] for p in prompts]
        job = f"{len(lens)} prompts of {min(lens)}-{max(lens)} tokens ({'+'.join(map(str, lens))}) split over the GPUs"
    elif scaling == "tp":
        job = f"one {prompts[0][0]}-token prompt per job, heads split over the GPUs"
    else:
        job = f"one {prompts[0][0]}-token prompt per GPU"
    return f"{name}: {arch} LLaMA (random init) sparse prefill, {job}, {mask_text(mask, topk)}"


def mask_cfg(name: str):
    """(mask builder parameters, pooled top-k) of a workload."""
    return (MASK_C4, 0) if name == "c4" else (MASK, TOPK)


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["c1", "c2", "c3", "c4", "c0"], default="c1")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-op16k", action="store_true", help="skip the 16K attention-op roofline record")
    ap.add_argument("--attn-only", action="store_true",
                    help="time the prefill attention kernel alone on one layer of the workload")
    ap.add_argument("--aux-op", choices=["mask", "token", "similarity"], default=None,
                    help="time one of the structure-side GPU paths on the workload's prompt (c1 shape)")
    ap.add_argument("--prefill-op", choices=["qkv"], default=None,
                    help="time the fused prefill q/k/v projection + RoPE + KV store + pooling against the "
                         "unfused sequence (three cuBLAS projections, then the RoPE/KV kernel) on one layer")
    ap.add_argument("--decode-op", choices=["dense", "sparse", "qkv"], default=None,
                    help="time the decode attention kernel alone on one layer of the workload: over every cached "
                         "block (dense) or over the last prompt row's list plus the generated blocks (sparse)")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# workload definition
# ---------------------------------------------------------------------------

def workload(name: str, rank: int, world: int):
    """Per-rank list of (prompt_len, seed) and the model architecture."""
    if name == "c1":
        return "1.3b", [(12288, 1000 + rank)], "weak"
    if name == "c3":
        return "6.7b", [(16384, 3000 + rank)], "weak"
    if name == "c4":
        # head-parallel: every rank works on the same prompt with its share of the heads
        return "33b", [(16384, 4000)], "tp"
    if name == "c2":
        import numpy as np
        from sabrecoder_b200.prompt_parallel import prompts_for_rank
        lens = np.random.default_rng(2).integers(12288, 16385, size=8).tolist()
        return "1.3b", [(int(lens[i]), 2000 + i) for i in prompts_for_rank(lens, rank, world)], "strong"
    return None, [(4096, 0)], "weak"


def build_model(arch: str, device, rank: int = 0, world: int = 1):
    """Random-init bf16 LLaMA of the named architecture. The 33B model is built
    on the meta device, split head-parallel for (rank, world) and only this
    rank's shard is given storage, so the full weights are never held."""
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(**ARCH[arch], head_dim=128, max_position_embeddings=16384, rope_theta=100000.0,
                      rope_scaling={"rope_type": "linear", "factor": 4.0}, rms_norm_eps=1e-6,
                      tie_word_embeddings=False, attn_implementation="sdpa")
    torch.manual_seed(0)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        if arch == "33b":
            from sabrecoder_b200 import tensor_parallel as TP
            with torch.device("meta"):
                model = LlamaForCausalLM(cfg)
            TP.shard_llama_(model, rank, world)
            TP.materialize_random_(model, device, seed=0)
        else:
            with torch.device(device):
                model = LlamaForCausalLM(cfg)
    finally:
        torch.set_default_dtype(prev)
    return model.eval(), cfg


def prompt_inputs(L: int, seed: int, vocab: int = 32256, mix=None):
    import numpy as np
    from sabrecoder_b200.spans import BENCH_SPAN_MIX, make_spans
    ids = np.random.default_rng(seed).integers(0, vocab, size=(1, L), dtype=np.int64)
    spans = make_spans(L, seed, **(BENCH_SPAN_MIX if mix is None else mix))
    return ids, spans


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------

class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sms, mx, reasons, power = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sms.append(float(p[1]))
                mx = float(p[2])
                power.append(float(p[3]))
            except ValueError:
                continue
            for nm, val in zip(names, p[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sms) if sms else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sms),
                "power_w_max": max(power) if power else None}


# ---------------------------------------------------------------------------
# profiles/ figures (ncu summary committed next to this script)
# ---------------------------------------------------------------------------

def profile_traffic(kernel_tag: str):
    """Per-launch DRAM bytes from the committed ncu summary, if present."""
    path = os.path.join(ROOT, "profiles", f"{kernel_tag}.md")
    if not os.path.exists(path):
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", open(path).read())
    return float(m.group(1)) if m else None


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        d = json.load(open(path))
        return d.get("bf16_tflops"), d.get("bf16_tflops_sustained"), d.get("hbm_gbs"), "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


# ---------------------------------------------------------------------------
# CPU side (reference arm and cpu_baseline)
# ---------------------------------------------------------------------------

def cpu_layer_sample(arch: str, L: int, seed: int, repeats: int = 1, mask=None, topk=None):
    """One decoder layer of the workload on the host cores with the reference's
    dense-masked attention arithmetic; returns (list of seconds per layer call,
    layers, threads). Structure lists and pooled top-k come from the oracle."""
    mix = C4_SPAN_MIX if mask is MASK_C4 else None
    mask = MASK if mask is None else mask
    topk = TOPK if topk is None else topk
    import numpy as np
    import torch
    from oracle import attention_oracle as AO
    from oracle import mask_oracle as MO
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaDecoderLayer, LlamaRotaryEmbedding
    torch.set_num_threads(os.cpu_count() or 1)
    threads = torch.get_num_threads()
    a = ARCH[arch]
    cfg = LlamaConfig(**a, head_dim=128, max_position_embeddings=16384, rope_theta=100000.0,
                      rope_scaling={"rope_type": "linear", "factor": 4.0}, rms_norm_eps=1e-6)
    torch.manual_seed(0)
    layer = LlamaDecoderLayer(cfg, 0).float().eval()
    rot = LlamaRotaryEmbedding(cfg)
    _, spans = prompt_inputs(L, seed, mix=mix)
    base = MO.build_block_mask_tokens(spans.token_to_chunk(), len(spans.spans), spans.import_chunks, spans.deps,
                                      spans.signature_token_mask(), seq_len=L, **mask).astype(bool)
    B = mask["block_size"]
    attn = layer.self_attn

    class DenseMasked(torch.nn.Module):
        def forward(self, hidden_states, position_embeddings=None, **kw):
            from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
            b, l = hidden_states.shape[:2]
            shp = (b, l, -1, 128)
            q = attn.q_proj(hidden_states).view(shp).transpose(1, 2)
            k = attn.k_proj(hidden_states).view(shp).transpose(1, 2)
            v = attn.v_proj(hidden_states).view(shp).transpose(1, 2)
            q, k = apply_rotary_pos_emb(q, k, *position_embeddings)
            grp = q.shape[1] // k.shape[1]
            if topk > 0:
                qm = MO.pooled_block_means(q.detach().numpy(), l, B)
                km = MO.pooled_block_means(k.detach().numpy(), l, B)
                ext = MO.topk_extend_mask(base, MO.pooled_scores(qm, km.repeat(grp, axis=1)), topk)
            else:
                ext = np.broadcast_to(base, (1, q.shape[1]) + base.shape)
            outs = []
            for h in range(q.shape[1]):  # one head at a time bounds host memory
                hk = h // grp
                outs.append(AO.dense_masked_sdpa(q[:, h:h + 1], k[:, hk:hk + 1], v[:, hk:hk + 1],
                                                 torch.from_numpy(np.ascontiguousarray(ext[0, h])), B))
            o = torch.cat(outs, 1).transpose(1, 2).reshape(b, l, -1)
            return attn.o_proj(o), None

    layer.self_attn = DenseMasked()
    x = torch.randn(1, L, a["hidden_size"], generator=torch.Generator().manual_seed(seed)) * 0.02
    pos = torch.arange(L).unsqueeze(0)
    dts = []
    with torch.no_grad():
        pe = rot(x, pos)
        for _ in range(repeats):
            t0 = time.perf_counter()
            layer(x, position_embeddings=pe, attention_mask=None)
            dts.append(time.perf_counter() - t0)
    return dts, a["num_hidden_layers"], threads


def cpu_model_ends(arch: str, L: int, seed: int) -> float:
    """Seconds of the model's parts outside the decoder layers on the host
    cores: token embedding of the prompt, rotary tables, the final RMSNorm and
    the LM head on the last position (the prefill keeps only its logits)."""
    import torch
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaRMSNorm, LlamaRotaryEmbedding
    a = ARCH[arch]
    cfg = LlamaConfig(**a, head_dim=128, max_position_embeddings=16384, rope_theta=100000.0,
                      rope_scaling={"rope_type": "linear", "factor": 4.0}, rms_norm_eps=1e-6)
    torch.manual_seed(0)
    emb = torch.nn.Embedding(a["vocab_size"], a["hidden_size"])
    norm = LlamaRMSNorm(a["hidden_size"], eps=1e-6)
    head = torch.nn.Linear(a["hidden_size"], a["vocab_size"], bias=False)
    rot = LlamaRotaryEmbedding(cfg)
    ids, _ = prompt_inputs(L, seed)
    ids = torch.from_numpy(ids)
    with torch.no_grad():
        t0 = time.perf_counter()
        h = emb(ids)
        rot(h, torch.arange(L).unsqueeze(0))
        head(norm(h)[:, -1:])
        return time.perf_counter() - t0


def run_reference_arm(args, rank, world):
    """The reference's CPU path on the host cores, on a bounded sample: each
    timed step is one decoder layer of the workload's first prompt (fp32,
    projections, RoPE, the reference's dense-masked attention per head, MLP),
    so `steps` and `ms_per_step` are the layer calls actually timed. The
    prompt's prefill time is then the mean layer time x the layer count plus
    the model's ends (embedding, final norm, LM head on the last position,
    timed once), and `value` = prompt tokens / that time."""
    if rank != 0:
        return
    arch, prompts, scaling = workload(args.workload, 0, 1)
    arch = arch or "1.3b"
    L, seed = prompts[0]
    mask, topk = mask_cfg(args.workload)
    nwarm = min(args.warmup, 1)
    dts, layers, threads = cpu_layer_sample(arch, L, seed, repeats=nwarm + args.steps, mask=mask, topk=topk)
    timed = dts[nwarm:]
    ends = cpu_model_ends(arch, L, seed)
    per_layer = statistics.mean(timed)
    per_prompt = per_layer * layers + ends
    value = L / per_prompt
    sample = (f"{len(timed)} timed calls of 1 of {layers} decoder layers (fp32, dense-masked SDPA per head) on one "
              f"{L}-token prompt, {per_layer:.3f} s each, x{layers} + {ends * 1e3:.1f} ms of embedding, final norm "
              f"and LM head = {per_prompt:.1f} s per prompt")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": len(timed), "warmup": nwarm, "ms_per_step": per_layer * 1e3, "higher_is_better": True,
        "scaling": "strong" if scaling == "tp" else scaling, "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload_text(args.workload), "seq_len": L, "global_batch": 1,
                   "step": "one decoder layer of one prompt (a bounded sample of the prefill)"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def run_ours(args, rank, world, dist):
    import numpy as np
    import torch
    from sabrecoder_b200 import kernels as K
    from sabrecoder_b200 import sabrecoder_llama as SL
    from sabrecoder_b200.sabrecoder_attention import StructureAwareMaskBuilder

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    arch, prompts, scaling = workload(args.workload, rank, world)
    if args.prefill_op == "qkv":
        return run_qkv_prefill_op(args, rank, world, dist)
    if args.decode_op == "qkv":
        return run_qkv_op(args, rank, world, dist)
    if args.decode_op:
        return run_decode_op(args, rank, world, dist)
    if args.aux_op:
        return run_aux_op(args, rank, world, dist)
    if arch is None or args.attn_only:
        return run_op_bench(args, rank, world, dist)
    mask, topk = mask_cfg(args.workload)
    tp = scaling == "tp"
    model, cfg = build_model(arch, dev, rank, world) if tp else build_model(arch, dev)
    SL.patch_model_with_sabrecoder_attention(model, None, topk_blocks=topk, verbose=False, **mask)
    mb = StructureAwareMaskBuilder(None, **mask)
    SL.set_current_code("<synthetic prompt>")

    prepared = []
    for L, seed in prompts:
        ids, spans = prompt_inputs(L, seed, cfg.vocab_size, mix=C4_SPAN_MIX if tp else None)
        bi, bc, bm = mb.build_block_indices_from_spans(spans, dev)
        prepared.append((L, torch.from_numpy(ids).to(dev), bi, bc, bm, ids, spans))
    tokens_per_step = sum(p[0] for p in prepared)
    # One preallocated KV cache, refilled by every prefill (the fused RoPE
    # kernel writes K/V rows straight into it).
    from sabrecoder_b200.kv_cache import SabreKVCache
    cache = SabreKVCache(cfg, batch_size=1, max_cache_len=max(p[0] for p in prepared) + 64, device=dev,
                         num_kv_heads=cfg.num_key_value_heads // (world if tp else 1))

    def step():
        for L, ids_d, bi, bc, bm, _, _ in prepared:
            SL.set_precomputed_blocks(bi, bc)
            cache.reset()
            model(input_ids=ids_d, past_key_values=cache, use_cache=True, logits_to_keep=1)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    with torch.no_grad():
        for _ in range(args.warmup):
            step()
        barrier()
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        phys = vis.split(",")[dev.index] if vis else str(dev.index)
        clocks = ClockSampler(int(phys) if phys.isdigit() else dev.index)
        clocks.start()
        events = K.set_prefill_timing(True)
        launches0 = K.LAUNCHES[0]
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        s.record()
        for _ in range(args.steps):
            step()
        e.record()
        barrier()
        K.set_prefill_timing(False)
        launches = K.LAUNCHES[0] - launches0
        ck = clocks.stop()
        ms = s.elapsed_time(e)
        # attention kernel: per-launch algorithmic FLOPs over event durations
        kt, kf, act, tot_blocks = 0.0, 0.0, 0.0, 0.0
        for a, b, cnt, heads, blk in events:
            kt += a.elapsed_time(b)
            n_active = float(cnt.sum().item()) * heads
            kf += n_active * 4 * blk * blk * 128
            nbq = cnt.shape[-1]
            act += n_active
            tot_blocks += (cnt.numel() // nbq) * heads * nbq * (nbq + 1) / 2
        nlaunch = max(len(events), 1)
        dens = []
        for L, _, bi, bc, bm, _, _ in prepared:
            nb = bm.shape[0]
            dens.append(float(bm.sum().item()) / (nb * (nb + 1) / 2))

    ms_max = ms
    if dist is not None:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = float(t.item())
    value = tokens_per_step * world * args.steps / (ms_max / 1e3) if scaling == "weak" else None
    if tp:  # every rank prefills the same prompt with its share of the heads
        value = tokens_per_step * args.steps / (ms_max / 1e3)
    if scaling == "strong":
        tot = torch.tensor([tokens_per_step], device=dev, dtype=torch.float64)
        if dist is not None:
            dist.all_reduce(tot)
        value = float(tot.item()) * args.steps / (ms_max / 1e3)

    # end to end through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        e2e = e2e_through_api(model, mb, prepared, args, dev, dist, cache)

    burst, sustained, hbm, which = measured_peaks()
    per_launch_flop = kf / nlaunch
    per_launch_ms = kt / nlaunch
    achieved = per_launch_flop / (per_launch_ms * 1e-3) / 1e12 if per_launch_ms > 0 else 0.0
    traffic = profile_traffic(f"prefill_bsa_{args.workload}")

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        L0, seed0 = prompts[0]
        dts, layers, threads = cpu_layer_sample(arch, L0, seed0, mask=mask, topk=topk)
        ends = cpu_model_ends(arch, L0, seed0)
        v = L0 / (dts[0] * layers + ends)
        cpu = {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port",
               "sample": f"1 of {layers} decoder layers (fp32, dense-masked SDPA per head) on {L0} tokens, "
                         f"scaled x{layers}, + embedding, final norm and LM head ({ends * 1e3:.1f} ms)"}

    # The 16K-token attention op the prefill target is stated for (the c3
    # layer shape: 32 heads, structure + top-8 lists), timed alone with L2
    # flushed, so every bench line carries a 16K roofline.
    roof16 = None
    if not args.no_op16k:
        ms16, flop16, dens16, H16, L16, iss16 = op_measure("c3", rank, max(3, min(args.steps, 10)), 3)
        ach16 = flop16 / ms16 / 1e9
        roof16 = {"kernel": "sabre prefill_bsa_kernel", "bound": "tensor",
                  "workload": f"attention op B=1 H={H16} L={L16} D=128 block 64, structure + top-{TOPK}, "
                              f"density {dens16:.4f}, {L2Flush.NOTE}",
                  "achieved": ach16, "peak": burst, "unit": "TFLOP/s", "frac": ach16 / burst,
                  "peak_kind": f"{which} bf16 dense, burst (kernel timed alone)",
                  "frac_of_sustained": ach16 / sustained, "flop_per_launch": flop16, "ms_per_launch": ms16,
                  "issued_flop_per_launch": iss16, "issued_tflops": iss16 / ms16 / 1e9,
                  "traffic": profile_traffic("prefill_bsa_c3_op")}

    weight_gb = sum(p.numel() * p.element_size() for p in model.parameters()) / 1e9
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "strong" if scaling == "tp" else scaling, "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": workload_text(args.workload),
                       "prompts_this_rank": "+".join(str(p[0]) for p in prepared),
                       "seq_len": prepared[0][0], "global_batch": len(prompts) * (world if scaling == "weak" else 1),
                       "parallelism": (f"head-parallel TP x{world} with sequence parallelism: NCCL reduce-scatter "
                                       f"after o_proj and down_proj, all-gather before attention and MLP"
                                       if tp and world > 1 else f"prompt-parallel x{world}, no collectives"),
                       "l2": f"inputs larger than L2 ({weight_gb:.1f} GB of weights read per step per GPU)",
                       "density_structure": round(statistics.mean(dens), 4),
                       "density_with_topk": round(act / tot_blocks, 4) if tot_blocks else None},
            "attn_tflops": kf / (kt * 1e-3) / 1e12 if kt > 0 else None,
            "attn_ms_per_step": kt / args.steps,
            "roofline": {"kernel": "sabre prefill_bsa_kernel", "bound": "tensor", "achieved": achieved,
                         "peak": sustained, "unit": "TFLOP/s", "frac": achieved / sustained if sustained else None,
                         "peak_kind": f"{which} bf16 dense, sustained (kernel timed inside a long step)",
                         "flop_per_launch": per_launch_flop, "ms_per_launch": per_launch_ms,
                         "traffic": traffic},
            "roofline_16k": roof16,
            "gpu_launches": launches,
            "clocks": ck,
            "e2e": e2e,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)


def e2e_through_api(model, mb, prepared, args, dev, dist, cache):
    """tokens/s through the user-facing calls, with host inputs: each step
    copies the prompt ids and the token-level structure from pinned host
    memory, builds the block lists on the GPU, runs the patched model and
    reads the last-position logits back."""
    import numpy as np
    import torch
    from sabrecoder_b200 import sabrecoder_llama as SL
    host = []
    for L, _, _, _, _, ids, spans in prepared:
        ptr, idx = spans.deps_csr()
        arrs = dict(ids=torch.from_numpy(ids).pin_memory(),
                    t2c=torch.from_numpy(spans.token_to_chunk()).pin_memory(),
                    flags=torch.tensor([1 if s.tag == "import" else 0 for s in spans.spans],
                                       dtype=torch.uint8).pin_memory(),
                    ptr=torch.from_numpy(ptr).pin_memory(), idx=torch.from_numpy(idx).pin_memory(),
                    gtm=torch.from_numpy(spans.signature_token_mask()).pin_memory())
        host.append((L, arrs))
    h2d = sum(sum(t.numel() * t.element_size() for t in a.values()) for _, a in host)
    d2h = 0

    def step():
        nonlocal d2h
        d2h = 0
        for L, a in host:
            d = {k: v.to(dev, non_blocking=True) for k, v in a.items()}
            bits, dense = mb.build_block_mask_tokens(d["t2c"], d["flags"], d["ptr"], d["idx"], d["gtm"], L, dev)
            bi, bc = mb._indices_from_bits(bits, dense.shape[0], 1)
            SL.set_precomputed_blocks(bi, bc)
            cache.reset()
            logits = model(input_ids=d["ids"], past_key_values=cache, use_cache=True, logits_to_keep=1).logits
            out = logits.to("cpu")
            d2h += out.numel() * out.element_size()

    with torch.no_grad():
        for _ in range(max(1, args.warmup)):
            step()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(args.steps):
            step()
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e)
    if dist is not None:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    toks = sum(L for L, _ in host)
    world = dist.get_world_size() if dist is not None else 1
    _, _, scaling = workload(args.workload, 0, world)
    if scaling == "weak":
        val = toks * world * args.steps / (ms / 1e3)
    elif scaling == "tp":  # all ranks prefill the same prompt
        val = toks * args.steps / (ms / 1e3)
    else:
        tt = torch.tensor([toks], device=dev, dtype=torch.float64)
        if dist is not None:
            dist.all_reduce(tt)
        val = float(tt.item()) * args.steps / (ms / 1e3)
    return {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}


class L2Flush:
    """Evicts the 126 MB L2 between timed launches by reading a 256 MB buffer
    (a sum into one scalar). Reading leaves only clean lines behind, so the
    timed kernel does not pay for writing back a flush buffer's dirty lines."""
    NOTE = "L2 flushed between iterations by reading a 256 MB buffer"

    def __init__(self, dev):
        import torch
        self.buf = torch.ones(64 * 1024 * 1024, dtype=torch.float32, device=dev)
        self.out = torch.empty((), dtype=torch.float32, device=dev)

    def __call__(self):
        import torch
        torch.sum(self.buf, dim=0, out=self.out)


OP_SHAPES = {"c0": (16, 4096, "spans"), "c1": (16, 12288, "bench"), "c2": (16, 16384, "bench"),
             "c3": (32, 16384, "bench")}


def issued_tile_flop(idx, cnt) -> float:
    """MMA work the prefill kernel issues for block-64 lists: a 128-row CTA
    runs S = Q K^T and P V over the union of its two 64-row query blocks'
    key tiles (listed, and not after the block), 4 x 128 x 64 x 128 FLOP per
    tile; the algorithmic count takes each block's own list only."""
    import torch
    _, H, nb, ma = idx.shape
    dev = idx.device
    pos = torch.arange(ma, device=dev).view(1, 1, ma)
    qb = torch.arange(nb, device=dev).view(1, nb, 1)
    kb = idx[0].long()
    valid = (pos < cnt[0].unsqueeze(-1)) & (kb >= 0) & (kb <= qb)
    m = torch.zeros(H, nb + (nb & 1), nb + 1, dtype=torch.bool, device=dev)
    m[:, :nb].scatter_(2, torch.where(valid, kb, torch.full_like(kb, nb)), True)
    tiles = m[..., :nb].view(H, -1, 2, nb).any(2).sum().item()
    return float(tiles) * 4 * 128 * 64 * 128


def op_measure(name: str, rank: int, steps: int, warmup: int):
    """The prefill attention op alone on one layer's shape of a workload
    (c0: B=1, H=16, L=4096; c1: H=16, L=12288; c3: H=32, L=16384), block 64,
    structure + pooled top-8 lists, L2 flushed between timed launches (the
    flush is outside the timed window). Returns (ms per launch, algorithmic
    FLOP per launch, density, H, L, issued FLOP per launch)."""
    import torch
    from sabrecoder_b200 import kernels as K
    from sabrecoder_b200.sabrecoder_attention import StructureAwareMaskBuilder
    from sabrecoder_b200.spans import BENCH_SPAN_MIX, make_spans
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    H, L, mix = OP_SHAPES[name]
    blk = 64
    g = torch.Generator(device=dev).manual_seed(rank)
    q, k, v = (torch.randn(1, L, H, 128, device=dev, generator=g, dtype=torch.bfloat16).transpose(1, 2)
               for _ in range(3))
    mb = StructureAwareMaskBuilder(None, **MASK)
    spans = make_spans(L, rank) if mix == "spans" else make_spans(L, 1000 + rank, **BENCH_SPAN_MIX)
    bi, bc, bm = mb.build_block_indices_from_spans(spans, dev)
    qm, km = K.pool_blocks(q, blk), K.pool_blocks(k, blk)
    idx, cnt, mx, _ = K.topk_extend(qm, km, mb.last_block_bits, TOPK)
    ma = int(mx.item())
    idx = idx[..., :ma].contiguous()
    out = torch.empty_like(q)
    flush = L2Flush(dev)
    for _ in range(warmup):
        K.prefill_bsa(q, k, v, idx, cnt, blk, out=out)
    torch.cuda.synchronize()
    tot = 0.0
    for _ in range(steps):
        flush()
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        s.record()
        K.prefill_bsa(q, k, v, idx, cnt, blk, out=out)
        e.record()
        torch.cuda.synchronize()
        tot += s.elapsed_time(e)
    ms = tot / steps
    flop = float(cnt.sum().item()) * 4 * blk * blk * 128
    nb = bm.shape[0]
    dens = float(cnt.sum().item()) / (H * nb * (nb + 1) / 2)
    return ms, flop, dens, H, L, issued_tile_flop(idx, cnt)


def run_op_bench(args, rank, world, dist):
    """The prefill attention op alone on one layer's shape of the workload."""
    ms, flop, dens, H, L, issued = op_measure(args.workload, rank, args.steps, args.warmup)
    burst, sustained, hbm, which = measured_peaks()
    traffic = profile_traffic(f"prefill_bsa_{args.workload}_op")
    if rank == 0:
        print(json.dumps({"metric": "effective sparse-attn TFLOP/s (single op)", "value": flop / ms / 1e9,
                          "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                          "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                          "dtype": "bf16", "data": "synthetic",
                          "config": {"workload": f"{args.workload} attention op: B=1 H={H} L={L} D=128 block 64, "
                                                 f"structure + top-{TOPK}, density {dens:.4f}",
                                     "l2": L2Flush.NOTE},
                          "roofline": {"kernel": "sabre prefill_bsa_kernel", "bound": "tensor",
                                       "achieved": flop / ms / 1e9, "peak": burst, "unit": "TFLOP/s",
                                       "frac": flop / ms / 1e9 / burst, "peak_kind": f"{which} bf16 dense, burst",
                                       "flop_per_launch": flop, "ms_per_launch": ms,
                                       "issued_flop_per_launch": issued, "issued_tflops": issued / ms / 1e9,
                                       "traffic": traffic}}))


def _events_ms(fn, steps, warmup):
    """Mean device time of fn() over `steps` calls (CUDA events on the current stream)."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    tot = 0.0
    for _ in range(steps):
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        tot += s.elapsed_time(e)
    return tot / steps


def _token_rule_from_spans(spans, mask):
    """Per-token arrays of the token-level rule for seeded spans (chunk,
    same-chunk group, global flag, dependency bits), as the builder derives
    them from text (prefix/suffix/import/signature tokens global)."""
    import numpy as np
    L = spans.seq_len
    t2c = spans.token_to_chunk().astype(np.int32)
    n = len(spans.spans)
    glob = spans.signature_token_mask().astype(bool)
    imp = np.zeros(max(n, 1), bool)
    for c in spans.import_chunks:
        imp[c] = True
    glob |= (t2c >= 0) & imp[np.clip(t2c, 0, max(n - 1, 0))]
    glob[:min(mask["num_prefix_tokens"], L)] = True
    glob[max(0, L - mask["num_suffix_tokens"]):] = True
    bpg = max(1, mask["max_chunk_tokens"] // 64)
    gidx = (np.arange(L) // 64) // bpg
    grp = (t2c.astype(np.int64) * (int(gidx.max()) + 2) + gidx).astype(np.int32)
    words = max((n + 31) // 32, 1)
    dep = np.zeros((max(n, 1), words), np.uint32)
    ptr, idx = spans.deps_csr()
    for a in range(n):
        for t in idx[ptr[a]:ptr[a + 1]]:
            dep[a, int(t) >> 5] |= np.uint32(1 << (int(t) & 31))
    return t2c, grp, glob.astype(np.uint8), dep, n


def run_aux_op(args, rank, world, dist):
    """Device time of a structure-side GPU path on the workload's prompt (one
    layer's c1 shape: 16 heads, 12288 tokens, block 64):
      mask        block mask (R0-R3) + index lists from token-level structure;
      token       token-level variant: block lists and per-block 64x64 masks
                  from the token rule, then the token-mask prefill kernel;
      similarity  chunk vectors (mean of 2048-wide bf16 embedding rows of the
                  chunk's tokens, up to 256) and each chunk's 8 most similar
                  chunks.
    The CPU leg times the oracle's restatement of the same step on a bounded
    sample (the whole step for mask/similarity, token rule at 2048 tokens)."""
    import numpy as np
    import torch
    from oracle import mask_oracle as MO
    from sabrecoder_b200 import kernels as K
    from sabrecoder_b200.sabrecoder_attention import StructureAwareMaskBuilder
    from sabrecoder_b200.spans import BENCH_SPAN_MIX, make_spans
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    H, L, _ = OP_SHAPES["c1"]
    spans = make_spans(L, 1000 + rank, **BENCH_SPAN_MIX)
    mb = StructureAwareMaskBuilder(None, **MASK)
    info, cpu = {}, None
    if args.aux_op == "mask":
        ptr, idx = spans.deps_csr()
        flags = np.asarray([1 if s.tag == "import" else 0 for s in spans.spans], np.uint8)
        d = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in
             dict(t2c=spans.token_to_chunk(), flags=flags, ptr=ptr, idx=idx, gtm=spans.signature_token_mask()).items()}

        def fn():
            bits, dense = mb.build_block_mask_tokens(d["t2c"], d["flags"], d["ptr"], d["idx"], d["gtm"], L, dev)
            K.indices_from_bits(bits, dense.shape[0])
        ms = _events_ms(fn, args.steps, args.warmup)
        t0 = time.perf_counter()
        MO.build_block_mask_tokens(spans.token_to_chunk(), len(spans.spans), spans.import_chunks, spans.deps,
                                   spans.signature_token_mask(), seq_len=L, **MASK)
        cpu = time.perf_counter() - t0
        value, unit, metric = ms * 1e3, "us", "block mask + index lists latency (one prompt)"
        info = {"chunks": len(spans.spans)}
    elif args.aux_op == "token":
        t2c, grp, glob, dep, n = _token_rule_from_spans(spans, MASK)
        up = lambda a, dt: torch.as_tensor(np.ascontiguousarray(a), dtype=dt).to(dev)
        tc, tg, tgl = up(t2c, torch.int32), up(grp, torch.int32), up(glob, torch.uint8)
        db = up(dep.view(np.int32), torch.int32)
        w = MASK["window_size"]
        built = {}

        def build():
            bits = K.token_block_mask(tc, tg, tgl, db, n, w)
            nb = bits.shape[0]
            idx, cnt, mx = K.indices_from_bits(bits, nb)
            lists = idx[:, :max(int(mx.item()), 1)].contiguous()
            built["l"], built["c"] = lists, cnt
            built["m"] = K.token_tile_masks(tc, tg, tgl, db, n, w, lists, cnt)
        ms_build = _events_ms(build, args.steps, args.warmup)
        g = torch.Generator(device=dev).manual_seed(rank)
        q, k, v = (torch.randn(1, L, H, 128, device=dev, generator=g, dtype=torch.bfloat16).transpose(1, 2)
                   for _ in range(3))
        bi, bc = built["l"][None], built["c"][None]
        out = torch.empty_like(q)
        flush = L2Flush(dev)

        def attn():
            flush()
            K.prefill_bsa(q, k, v, bi, bc, 64, out=out, token_masks=built["m"])
        ms_attn = _events_ms(attn, args.steps, args.warmup)
        ms_flush = _events_ms(flush, args.steps, 1)
        ms_attn = max(ms_attn - ms_flush, 1e-6)
        flop = float(bc.sum().item()) * H * 4 * 64 * 64 * 128
        Ls = 2048
        sp = make_spans(Ls, 1000 + rank, **BENCH_SPAN_MIX)
        t0 = time.perf_counter()
        MO.token_level_mask_tokens(sp.token_to_chunk(), len(sp.spans), sp.import_chunks, sp.deps,
                                   sp.signature_token_mask(), seq_len=Ls, **MASK)
        cpu = (time.perf_counter() - t0) * (L / Ls) ** 2  # O(L^2): scaled to the full prompt
        value, unit, metric = ms_build * 1e3, "us", "token-level lists + 64x64 masks latency (one prompt)"
        info = {"prefill_token_mode_tflops": flop / ms_attn / 1e9, "prefill_ms": ms_attn,
                "listed_pairs": int(bc.sum().item()), "density": float(bc.sum().item()) / (
                    (L // 64) * (L // 64 + 1) / 2)}
    else:
        n_chunks = len(spans.spans)
        ids = np.random.default_rng(rank).integers(0, 32256, size=L).astype(np.int32)
        tok_lists = [ids[s.start:s.end + 1][:256] for s in spans.spans]
        ptr = np.concatenate([[0], np.cumsum([len(t) for t in tok_lists])]).astype(np.int32)
        flat = np.concatenate(tok_lists).astype(np.int32)
        emb = (torch.randn(32256, 2048, generator=torch.Generator().manual_seed(5)) * 0.02).to(torch.bfloat16).to(dev)
        dptr, dflat = torch.from_numpy(ptr).to(dev), torch.from_numpy(flat).to(dev)
        rows = torch.arange(n_chunks, dtype=torch.int32, device=dev)
        kk = min(8, int(n_chunks * 0.1))

        def fn():
            vecs = K.chunk_vectors(emb, dptr, dflat)
            K.similarity_topk(vecs, rows, rows, rows, rows, kk)
        ms = _events_ms(fn, args.steps, args.warmup)
        e32 = emb.float().cpu().numpy()
        t0 = time.perf_counter()
        vec = MO.chunk_vectors_f16(e32, [t.tolist() for t in tok_lists])
        MO.similarity_topk(vec, list(range(n_chunks)), list(range(n_chunks)), list(range(n_chunks)),
                           list(range(n_chunks)), kk)
        cpu = time.perf_counter() - t0
        value, unit, metric = ms * 1e3, "us", "chunk-similarity vectors + top-k latency (one prompt)"
        info = {"chunks": n_chunks, "k": kk, "embedding": "32256 x 2048 bf16"}
    if rank == 0:
        print(json.dumps({"metric": metric, "value": value, "unit": unit, "n_gpus": 1, "steps": args.steps,
                          "warmup": args.warmup, "ms_per_step": value / 1e3, "higher_is_better": False,
                          "scaling": "weak", "vs_baseline": None, "dtype": "int32/bf16", "data": "synthetic",
                          "config": {"workload": f"{args.aux_op} on the c1 prompt (12288 tokens, 16 heads, block 64)",
                                     **info},
                          "cpu_baseline": {"value": cpu * 1e6, "unit": "us", "cores": 1, "kind": "port",
                                           "sample": "the oracle's restatement on the host"}}))


# (query heads, KV heads, prompt tokens, generated tokens) of one layer on one GPU.
DECODE_SHAPES = {"c0": (16, 16, 4096, 64), "c1": (16, 16, 12288, 64), "c2": (16, 16, 16384, 64),
                 "c3": (32, 32, 16384, 128), "c4": (56, 8, 16384, 64)}


# hidden size of each workload's model (query / KV heads come from DECODE_SHAPES).
HIDDEN = {"c0": 2048, "c1": 2048, "c2": 2048, "c3": 4096, "c4": 7168}


def run_qkv_op(args, rank, world, dist):
    """One decode token's q/k/v projection + rotary + KV store on one layer's
    shape (B=1): the fused kernel against the unfused sequence (three cuBLAS
    projections, then the RoPE + KV-store kernel). Bytes counted: the three
    weight matrices (the rest is a few KB).

    A decode step runs this once per layer on that layer's weights, so the
    headline times one CUDA-graph replay of `nlayer` calls over distinct weight
    sets (>= 1 GiB in total, several times the L2: every call reads its weights
    from HBM), per-call time = replay time / nlayer; `single_call` keeps the
    one-call figures with L2 flushed before them."""
    import torch
    from sabrecoder_b200 import kernels as K
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    Hq, Hkv, L, _ = DECODE_SHAPES[args.workload]
    hidden, D, T = HIDDEN[args.workload], 128, L + 64
    g = torch.Generator(device=dev).manual_seed(rank)
    x = torch.randn(1, hidden, device=dev, generator=g, dtype=torch.bfloat16)
    nbytes = (Hq + 2 * Hkv) * D * hidden * 2
    nlayer = max(4, -(-(1 << 30) // nbytes))
    ws = [[torch.randn(h * D, hidden, device=dev, generator=g, dtype=torch.bfloat16) / hidden ** 0.5
           for h in (Hq, Hkv, Hkv)] for _ in range(nlayer)]
    cos = torch.randn(1, D, device=dev, generator=g, dtype=torch.bfloat16)
    sin = torch.randn(1, D, device=dev, generator=g, dtype=torch.bfloat16)
    kc = torch.zeros(1, Hkv, T, D, device=dev, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    q = torch.empty(1, Hq, D, device=dev, dtype=torch.bfloat16)
    pos = L

    def fused(w):
        K.qkv_rope_decode(x, *w, cos, sin, q, kc, vc, pos)

    def unfused(w):
        qq = torch.nn.functional.linear(x, w[0]).view(1, 1, Hq, D)
        kk = torch.nn.functional.linear(x, w[1]).view(1, 1, Hkv, D)
        vv = torch.nn.functional.linear(x, w[2]).view(1, 1, Hkv, D)
        K.rope_qkv(qq, kk, vv, cos.view(1, 1, D), sin.view(1, 1, D), kc, vc, pos0=pos)

    def graph_of(fn, sets):
        for _ in range(max(3, args.warmup)):
            for w in sets:
                fn(w)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            with torch.cuda.graph(graph, stream=side):
                for w in sets:
                    fn(w)
        torch.cuda.current_stream().wait_stream(side)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        return graph

    def timed(graph, flush=None):
        tot = 0.0
        for _ in range(args.steps):
            if flush is not None:
                flush()
            s, e = torch.cuda.Event(True), torch.cuda.Event(True)
            s.record()
            graph.replay()
            e.record()
            torch.cuda.synchronize()
            tot += s.elapsed_time(e)
        return tot / args.steps

    flush = L2Flush(dev)
    times, single = {}, {}
    for name, fn in (("fused", fused), ("unfused", unfused)):
        gr = graph_of(fn, ws)
        times[name] = timed(gr) / nlayer
        del gr
        gr = graph_of(fn, ws[:1])
        single[name] = timed(gr, flush)
        del gr
    gbs = nbytes / times["fused"] / 1e6
    _, _, hbm, which = measured_peaks()
    if rank == 0:
        print(json.dumps({"metric": "decode q/k/v projection + rotary + KV store GB/s (single op)", "value": gbs,
                          "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                          "ms_per_step": times["fused"], "higher_is_better": True, "scaling": "weak",
                          "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                          "config": {"workload": f"{args.workload} decode q/k/v: B=1 hidden={hidden} Hq={Hq} "
                                                 f"Hkv={Hkv}; {nlayer} calls per replay, one per layer's weights",
                                     "l2": f"{nlayer} distinct {nbytes / 1e6:.1f} MB weight sets per replay "
                                           f"({nlayer * nbytes / 1e9:.2f} GB): each call reads its weights from HBM",
                                     "unfused_ms": times["unfused"]},
                          "single_call": {"fused_ms": single["fused"], "unfused_ms": single["unfused"],
                                          "l2": L2Flush.NOTE},
                          "roofline": {"kernel": "sabre qkv_rope_decode_kernel", "bound": "hbm", "achieved": gbs,
                                       "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                                       "peak_kind": f"{which} HBM copy bandwidth", "bytes_per_launch": nbytes,
                                       "ms_per_launch": times["fused"], "traffic": None}}))


# (hidden, query heads, KV heads, prompt tokens) of one prefill layer on one GPU.
PREFILL_QKV_SHAPES = {"c1": (2048, 16, 16, 12288), "c3": (4096, 32, 32, 16384), "c4": (7168, 56, 8, 16384)}


def run_qkv_prefill_op(args, rank, world, dist):
    """One prompt's q/k/v projection + RoPE + KV store (+ pooling by 64 when the
    workload uses the pooled top-k) on one layer's shape: the fused kernel
    (sabre_qkv_proj_rope) against the unfused sequence (three cuBLAS
    projections, then sabre_rope_qkv), L2 flushed between launches. FLOPs
    counted: the projection, 2 x L x N x hidden."""
    import torch
    from sabrecoder_b200 import kernels as K
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    hidden, Hq, Hkv, L = PREFILL_QKV_SHAPES.get(args.workload, PREFILL_QKV_SHAPES["c1"])
    _, topk = mask_cfg(args.workload)
    pool = 64 if topk else 0
    D = 128
    N = (Hq + 2 * Hkv) * D
    g = torch.Generator(device=dev).manual_seed(rank)
    x = (torch.randn(1, L, hidden, device=dev, generator=g) * 0.5).to(torch.bfloat16)
    w = (torch.randn(N, hidden, device=dev, generator=g) / hidden ** 0.5).to(torch.bfloat16)
    wq, wk, wv = w[:Hq * D], w[Hq * D:(Hq + Hkv) * D], w[(Hq + Hkv) * D:]
    ang = torch.rand(1, L, D // 2, device=dev, generator=g) * 50
    emb = torch.cat([ang, ang], -1)
    cos, sin = emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)
    kc = torch.zeros(1, Hkv, L + 64, D, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    q_out = torch.empty(1, L, Hq, D, dtype=torch.bfloat16, device=dev)

    def fused():
        K.qkv_proj_rope(x, w, cos, sin, q_out, kc, vc, pool_block=pool)

    def unfused():
        q = torch.nn.functional.linear(x, wq).view(1, L, Hq, D)
        k = torch.nn.functional.linear(x, wk).view(1, L, Hkv, D)
        v = torch.nn.functional.linear(x, wv).view(1, L, Hkv, D)
        K.rope_qkv(q, k, v, cos, sin, kc, vc, pool_block=pool)

    flush = L2Flush(dev)
    times = {}
    for name, fn in (("fused", fused), ("unfused", unfused), ("fused2", fused), ("unfused2", unfused)):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize()
        tot = 0.0
        for _ in range(args.steps):
            flush()
            s, e = torch.cuda.Event(True), torch.cuda.Event(True)
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize()
            tot += s.elapsed_time(e)
        times[name] = tot / args.steps
    tf = min(times["fused"], times["fused2"])
    tu = min(times["unfused"], times["unfused2"])
    flop = 2.0 * L * N * hidden
    burst, sustained, hbm, which = measured_peaks()
    ach = flop / tf / 1e9
    if rank == 0:
        print(json.dumps({"metric": "prefill q/k/v projection + rotary + KV store TFLOP/s (single op)", "value": ach,
                          "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                          "ms_per_step": tf, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                          "dtype": "bf16", "data": "synthetic",
                          "config": {"workload": f"{args.workload} prefill q/k/v: L={L} hidden={hidden} Hq={Hq} "
                                                 f"Hkv={Hkv}, pooling {'by 64' if pool else 'off'}",
                                     "l2": L2Flush.NOTE, "fused_ms": tf, "unfused_ms": tu,
                                     "gain_ms_per_layer": tu - tf, "runs_ms": times},
                          "roofline": {"kernel": "sabre qkv_proj_rope_kernel", "bound": "tensor", "achieved": ach,
                                       "peak": burst, "unit": "TFLOP/s", "frac": ach / burst,
                                       "peak_kind": f"{which} bf16 dense, burst", "flop_per_launch": flop,
                                       "ms_per_launch": tf, "traffic": None}}))


def run_decode_op(args, rank, world, dist):
    """The decode attention op on one layer's shape of the workload: one
    query row per head after a prompt of L tokens and `gen` generated tokens
    (c1: H=16, L=12288, 64 generated; c3: H=32, L=16384, 128 generated; c4:
    56 query heads over 8 KV heads, L=16384, block 128, 64 generated), K/V
    caches in HBM. Bytes counted are the K and V rows of the listed blocks
    (plus q and o).

    A decode step calls the op once per layer, each call on its own layer's
    cache. The headline number times that: one CUDA-graph replay of
    `ncache` consecutive calls over distinct caches (their total is several
    times the L2, so every call reads its cache from HBM), per-call time =
    replay time / ncache. `single_call` keeps the one-call figure (L2
    flushed before it), which carries the fixed cost of an event-timed
    launch (an empty kernel measures ~6 us that way on B200)."""
    import torch
    from sabrecoder_b200 import kernels as K
    from sabrecoder_b200.sabrecoder_attention import StructureAwareMaskBuilder
    from sabrecoder_b200.spans import BENCH_SPAN_MIX, make_spans
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    Hq, H, L, gen = DECODE_SHAPES[args.workload]
    mask, _ = mask_cfg(args.workload)
    blk = mask["block_size"]
    T = L + gen
    g = torch.Generator(device=dev).manual_seed(rank)
    cache_bytes = 2 * H * T * 128 * 2
    ncache = max(4, -(-(1 << 30) // cache_bytes))   # >= 1 GiB of caches, >= 8x the L2
    caches = [(torch.randn(1, H, T, 128, device=dev, generator=g, dtype=torch.bfloat16),
               torch.randn(1, H, T, 128, device=dev, generator=g, dtype=torch.bfloat16)) for _ in range(ncache)]
    q = torch.randn(1, Hq, 128, device=dev, generator=g, dtype=torch.bfloat16)
    nbk = (T + blk - 1) // blk
    if args.decode_op == "dense":
        lst = torch.arange(nbk, device=dev, dtype=torch.int32).unsqueeze(0)
        cnt = torch.tensor([nbk], dtype=torch.int32, device=dev)
    else:
        mb = StructureAwareMaskBuilder(None, **mask)
        mix = C4_SPAN_MIX if mask is MASK_C4 else BENCH_SPAN_MIX
        bi, bc, _ = mb.build_block_indices_from_spans(make_spans(L, 1000 + rank, **mix), dev)
        nb_p = (L + blk - 1) // blk
        c_last = int(bc[0, nb_p - 1].item())
        lst = torch.cat([bi[0, nb_p - 1, :c_last].to(torch.int32),
                         torch.arange(nb_p, nbk, device=dev, dtype=torch.int32)]).unsqueeze(0).contiguous()
        cnt = torch.tensor([lst.shape[1]], dtype=torch.int32, device=dev)
    seq = torch.tensor([T], dtype=torch.int32, device=dev)
    ws = torch.empty(K.decode_workspace_bytes(1, Hq, H, 128, lst.shape[1]), dtype=torch.uint8, device=dev)
    outs = [torch.empty_like(q) for _ in range(ncache)]

    def step(which):
        for i in which:
            kc, vc = caches[i]
            K.decode_bsa(q, kc, vc, lst, cnt, seq, blk, out=outs[i], workspace=ws)

    def graph_of(which):
        for _ in range(max(3, args.warmup)):
            step(which)
        torch.cuda.synchronize()
        # Replayed from a CUDA graph so the host-side argument handling of the
        # Python calls cannot leak into the device-timed window.
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            with torch.cuda.graph(graph, stream=side):
                step(which)
        torch.cuda.current_stream().wait_stream(side)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        return graph

    def timed(graph, flush=None):
        tot = 0.0
        for _ in range(args.steps):
            if flush is not None:
                flush()
            s, e = torch.cuda.Event(True), torch.cuda.Event(True)
            s.record()
            graph.replay()
            e.record()
            torch.cuda.synchronize()
            tot += s.elapsed_time(e)
        return tot / args.steps

    seq_graph = graph_of(range(ncache))
    ms = timed(seq_graph) / ncache
    one_graph = graph_of([0])
    ms1 = timed(one_graph, L2Flush(dev))
    rows = 0
    for kb in lst[0, :int(cnt.item())].tolist():
        rows += max(0, min(blk, T - kb * blk))
    nbytes = rows * H * 128 * 2 * 2 + 2 * Hq * 128 * 2
    gbs = nbytes / ms / 1e6
    _, _, hbm, which = measured_peaks()
    gqa = Hq // H >= 3  # the tensor-core kernel serves groups of three or more query heads per KV head
    traffic = profile_traffic(f"{'decode_gqa' if gqa else 'decode_bsa'}_{args.workload}_{args.decode_op}")
    kern = ("sabre decode_gqa_kernel + decode_combine_kernel" if gqa
            else "sabre decode_bulk_kernel + decode_combine_kernel")
    if rank == 0:
        print(json.dumps({"metric": "decode attention GB/s (single op)", "value": gbs, "unit": "GB/s",
                          "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                          "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                          "data": "synthetic",
                          "config": {"workload": f"{args.workload} decode op: B=1 Hq={Hq} Hkv={H} cache {T} tokens D=128 "
                                                 f"block {blk}, {args.decode_op} list of {int(cnt.item())} blocks; "
                                                 f"{ncache} calls per replay, one per layer cache",
                                     "l2": f"{ncache} distinct {cache_bytes / 1e6:.0f} MB caches per replay "
                                           f"({ncache * cache_bytes / 1e9:.2f} GB, > 8x L2): each call reads its "
                                           f"cache from HBM"},
                          "single_call": {"ms": ms1, "gbs": nbytes / ms1 / 1e6, "frac": nbytes / ms1 / 1e6 / hbm,
                                          "l2": L2Flush.NOTE},
                          "roofline": {"kernel": kern, "bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s",
                                       "frac": gbs / hbm, "peak_kind": f"{which} HBM copy bandwidth",
                                       "bytes_per_launch": nbytes, "ms_per_launch": ms, "traffic": traffic}}))


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    dist = None
    if args.impl == "reference":
        return run_reference_arm(args, rank, world)
    import torch
    if world > 1:
        import datetime

        import torch.distributed as tdist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                 device_id=torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0))))
        dist = tdist
    try:
        run_ours(args, rank, world, dist)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
