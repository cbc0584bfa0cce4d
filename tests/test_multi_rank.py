"""Multi-process host logic on CPU (gloo, world size 2): the prompt-parallel
split and gather, max-over-ranks timing, and head-parallel tensor
parallelism of a small LLaMA whose sharded forward (two all-reduces per
layer) must reproduce the unsharded model's logits."""

import datetime
import json
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from sabrecoder_b200 import prompt_parallel as PP
from sabrecoder_b200 import tensor_parallel as TP


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    return dist


# ---------------------------------------------------------------------------
# prompt-parallel split
# ---------------------------------------------------------------------------

def test_assign_prompts_lpt_properties():
    rng = np.random.default_rng(0)
    for world in (1, 2, 3, 4, 8):
        lens = rng.integers(12288, 16385, size=8).tolist()
        parts = PP.assign_prompts(lens, world)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(8))
        loads = PP.rank_loads(lens, world)
        # LPT bound: makespan <= mean load + the largest prompt
        assert max(loads) <= sum(lens) / world + max(lens)
        assert PP.assign_prompts(lens, world) == parts  # deterministic
    assert PP.assign_prompts([5, 5, 5, 5], 2) == [[0, 2], [1, 3]]
    assert PP.assign_prompts([], 3) == [[], [], []]
    with pytest.raises(ValueError):
        PP.assign_prompts([1], 0)
    with pytest.raises(ValueError):
        PP.prompts_for_rank([1, 2], 2, 2)


def _prompt_density(i: int) -> float:
    """Per-prompt work of the test: the structure mask density of a seeded prompt."""
    from oracle import mask_oracle as MO
    from sabrecoder_b200.spans import make_spans
    L = 1024 + 256 * i
    sp = make_spans(L, 50 + i)
    m = MO.build_block_mask_tokens(sp.token_to_chunk(), len(sp.spans), sp.import_chunks, sp.deps,
                                   sp.signature_token_mask(), seq_len=L, block_size=64, window_size=192,
                                   num_prefix_tokens=64, num_suffix_tokens=128, max_chunk_tokens=128,
                                   global_last_k_chunks=0)
    nb = m.shape[-1]
    return float(m.sum()) / (nb * (nb + 1) / 2)


def _pp_worker(rank, world, port, out_dir):
    dist = _init(rank, world, port)
    try:
        lens = [1024 + 256 * i for i in range(5)]
        res = PP.run_prompts(_prompt_density, lens, rank, world, dist=dist)
        t = PP.max_over_ranks(1.0 + rank, dist)
        with open(os.path.join(out_dir, f"pp{rank}.json"), "w") as f:
            json.dump({"res": res, "t": t, "mine": PP.prompts_for_rank(lens, rank, world)}, f)
    finally:
        dist.destroy_process_group()


def test_prompt_parallel_gloo_world2(tmp_path):
    port = _free_port()
    mp.spawn(_pp_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    r0 = json.load(open(tmp_path / "pp0.json"))
    r1 = json.load(open(tmp_path / "pp1.json"))
    want = [_prompt_density(i) for i in range(5)]
    assert r0["res"] == want          # gathered on rank 0 in prompt order
    assert r1["res"] is None
    assert r0["t"] == r1["t"] == 2.0  # max over ranks
    assert sorted(r0["mine"] + r1["mine"]) == list(range(5))
    assert not set(r0["mine"]) & set(r1["mine"])


# ---------------------------------------------------------------------------
# head-parallel tensor parallelism
# ---------------------------------------------------------------------------

def _tiny_cfg():
    from transformers import LlamaConfig
    return LlamaConfig(vocab_size=97, hidden_size=256, intermediate_size=384, num_hidden_layers=2,
                       num_attention_heads=4, num_key_value_heads=2, head_dim=64, max_position_embeddings=1024,
                       rope_theta=100000.0, rms_norm_eps=1e-6, attn_implementation="eager")


def _tiny_model():
    from transformers import LlamaForCausalLM
    torch.manual_seed(7)
    return LlamaForCausalLM(_tiny_cfg()).float().eval()


def _tiny_inputs(L=320):
    from oracle import mask_oracle as MO
    from sabrecoder_b200.spans import make_spans
    blk = 64
    sp = make_spans(L, 11)
    m = MO.build_block_mask_tokens(sp.token_to_chunk(), len(sp.spans), sp.import_chunks, sp.deps,
                                   sp.signature_token_mask(), seq_len=L, block_size=blk, window_size=64,
                                   num_prefix_tokens=64, num_suffix_tokens=64, max_chunk_tokens=128,
                                   global_last_k_chunks=0)
    idx, cnt = MO.block_indices_from_mask(m[None].astype(bool))
    ids = torch.from_numpy(np.random.default_rng(3).integers(0, 97, size=(1, L)))
    return ids, torch.from_numpy(idx), torch.from_numpy(cnt), blk


def _logits(model, ids, bi, bc, blk):
    from oracle.llama_oracle import patch_oracle
    patch_oracle(model, bi, bc, blk)
    with torch.no_grad():
        return model(input_ids=ids, use_cache=False).logits


def _batched(L, batch):
    ids, bi, bc, blk = _tiny_inputs(L)
    if batch == 2:  # a second, different prompt with the same lists
        ids = torch.cat([ids, ids.flip(1)], 0)
        bi, bc = bi.expand(2, -1, -1).contiguous(), bc.expand(2, -1).contiguous()
    return ids, bi, bc, blk


def _tp_worker(rank, world, port, out_dir, seq_par, L, batch):
    dist = _init(rank, world, port)
    try:
        model = _tiny_model()
        TP.shard_llama_(model, rank, world, sequence_parallel=seq_par)
        attn = model.model.layers[0].self_attn
        assert attn.q_proj.weight.shape[0] == 4 // world * 64
        assert attn.k_proj.weight.shape[0] == 2 // world * 64
        ids, bi, bc, blk = _batched(L, batch)
        out = _logits(model, ids, bi, bc, blk)
        if seq_par:
            # L even: the forward ran sequence-parallel; odd: all-reduces.
            assert model._sabre_sp.active == (L % world == 0)
        torch.save(out, os.path.join(out_dir, f"tp{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("seq_par,L,batch", [(False, 320, 1), (True, 320, 1), (True, 317, 1), (True, 320, 2)])
def test_tensor_parallel_gloo_world2_matches_unsharded(tmp_path, seq_par, L, batch):
    """Head-parallel logits equal the unsharded model's: with all-reduces, with
    the token-wise work split over the ranks (sequence parallel, length
    divisible by the ranks) and with an odd length (falls back to
    all-reduces), for one prompt and for a batch of two."""
    ids, bi, bc, blk = _batched(L, batch)
    ref = _logits(_tiny_model(), ids, bi, bc, blk)
    port = _free_port()
    mp.spawn(_tp_worker, args=(2, port, str(tmp_path), seq_par, L, batch), nprocs=2, join=True)
    for r in range(2):
        out = torch.load(tmp_path / f"tp{r}.pt")
        torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-4)


def test_tp_shapes_33b_and_uneven():
    from transformers import LlamaConfig
    c = LlamaConfig(hidden_size=7168, intermediate_size=19200, num_attention_heads=56, num_key_value_heads=8,
                    head_dim=128, num_hidden_layers=62, vocab_size=32256)
    assert TP.tp_shapes(c, 8) == (7, 1, 2400)
    assert TP.tp_shapes(c, 2) == (28, 4, 9600)
    with pytest.raises(ValueError):
        TP.tp_shapes(c, 16)  # 8 KV heads do not split over 16 ranks


def test_meta_build_and_materialize_sharded():
    """The 33B-shaped layers can be built on the meta device, sharded and given
    storage without materialising the full weights (checked on a 2-layer cut)."""
    from transformers import LlamaConfig, LlamaForCausalLM
    c = LlamaConfig(hidden_size=7168, intermediate_size=19200, num_attention_heads=56, num_key_value_heads=8,
                    head_dim=128, num_hidden_layers=2, vocab_size=256, max_position_embeddings=4096)
    with torch.device("meta"):
        m = LlamaForCausalLM(c)
    TP.shard_llama_(m, 3, 8)
    TP.materialize_random_(m, torch.device("cpu"), seed=1, dtype=torch.float32)
    attn = m.model.layers[1].self_attn
    assert tuple(attn.q_proj.weight.shape) == (7 * 128, 7168)
    assert tuple(attn.o_proj.weight.shape) == (7168, 7 * 128)
    assert tuple(m.model.layers[0].mlp.down_proj.weight.shape) == (7168, 2400)
    assert all(p.device.type == "cpu" for p in m.parameters())
    assert m.model.rotary_emb.inv_freq.device.type == "cpu"
    with torch.no_grad():
        out = m(input_ids=torch.arange(8)[None], use_cache=False).logits
    assert torch.isfinite(out).all()


# ---------------------------------------------------------------------------
# a rank that leaves
# ---------------------------------------------------------------------------

LEAVE_TIMEOUT_S = 5


def _leave_worker(rank, world, port, out_dir, seq_par, mode):
    """Rank 1 joins the group, then leaves before the first collective of
    the sharded forward: it exits ("exit") or stays alive without ever
    joining the collective ("stall"). Rank 0 runs the forward and records
    the error it gets and how long it took."""
    import time

    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=LEAVE_TIMEOUT_S))
    if rank == 1:
        if mode == "exit":
            os._exit(0)
        time.sleep(LEAVE_TIMEOUT_S + 3)
        os._exit(0)
    model = _tiny_model()
    TP.shard_llama_(model, rank, world, sequence_parallel=seq_par)
    ids, bi, bc, blk = _batched(320, 1)
    t0 = time.monotonic()
    try:
        _logits(model, ids, bi, bc, blk)
        res = {"error": None}
    except Exception as e:  # the collective's failure, whatever its type
        res = {"error": f"{type(e).__name__}: {str(e)[:300]}"}
    res["elapsed"] = time.monotonic() - t0
    with open(os.path.join(out_dir, "leave0.json"), "w") as f:
        json.dump(res, f)
    # The group is broken: leave without a collective teardown.
    os._exit(0)


@pytest.mark.parametrize("seq_par,mode", [(False, "stall"), (True, "stall"), (False, "exit")])
def test_tensor_parallel_survivor_gets_an_error_when_a_rank_leaves(tmp_path, seq_par, mode):
    """A rank that leaves between steps (exits, or stops taking part) makes
    the survivor's next head-parallel collective -- the all-reduce after
    o_proj, or the sequence-parallel all-gather before attention -- end with
    an error within the process group's timeout instead of waiting for
    ever."""
    port = _free_port()
    mp.spawn(_leave_worker, args=(2, port, str(tmp_path), seq_par, mode), nprocs=2, join=True)
    res = json.load(open(tmp_path / "leave0.json"))
    assert res["error"] is not None, res
    assert res["elapsed"] < LEAVE_TIMEOUT_S + 20, res
