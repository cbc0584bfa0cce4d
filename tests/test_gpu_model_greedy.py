"""Greedy tokens of the patched 1.3B model against the oracle model.

The deepseek-coder-1.3B architecture (24 layers, hidden 2048, 16 heads x 128,
MLP 5504, vocab 32256, RoPE theta 1e5 linear x4), random-init bf16 weights, a
12288-token prompt with the benchmark's structure spans and mask parameters,
block-sparse prefill with the structure lists (the reference's configuration:
no top-k extension) and dense decode, as the reference's evaluator runs it
(methods/sabrecoder/run_eval.py:340-348; wrapper
sabrecoder_llama_triton.py:270-319, dense decode :305-308).

The patched model generates 32 greedy tokens free-running on the GPU (its own
token is fed back every step, through the preallocated cache). The oracle
model is then run over that sequence (prompt plus our tokens), so at every
step it sees the same prefix, twice on the host with the same weights:

* in fp32 (weights widened exactly, the oracle's attention in fp32): the
  exact reference, against which both bf16 computations are measured;
* in bf16, the way the reference itself runs the model: its distance from
  the fp32 run is the reference's own bf16 rounding noise on this model.

Random-init weights give top-1/top-2 logit margins down to ~1e-3 (logit scale
~3), below the bf16 noise of any implementation, so an exact greedy choice
can only be asked for where the margin exceeds that noise. At every step:

* our logits are within NOISE_FACTOR x the reference's own bf16 noise of
  the exact logits (largest absolute difference over the vocabulary, the
  noise taken as its largest value over the 32 steps), and
* our token is the exact greedy choice, or the exact logits score it within
  that bound of their top-1 (a tie at bf16 precision).

Where every step is the exact greedy choice, the exact model's free-running
greedy sequence equals ours. The test prints the first step where the
choices differ (if any), the exact margin there, the smallest and median
margins, the logit errors, and how often the reference's own bf16 run
departs from the exact greedy choice on the same prefixes. Both LM heads
compute in fp32, so rounding logits to bf16 cannot create exact ties.
"""

import copy

import pytest
import torch

import bench

pytestmark = pytest.mark.gpu

STEPS = 32
PROMPT = 12288
NOISE_FACTOR = 2.0


def _fp32_head(model):
    model.lm_head.float()
    model.lm_head.register_forward_pre_hook(lambda mod, args: (args[0].float(),))


@pytest.mark.timeout(1800)
def test_greedy_tokens_match_oracle_on_1p3b_at_12k():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from oracle.llama_oracle import patch_oracle
    from sabrecoder_b200 import sabrecoder_llama as SL
    from sabrecoder_b200.kv_cache import SabreKVCache
    from sabrecoder_b200.sabrecoder_attention import StructureAwareMaskBuilder
    from transformers import DynamicCache

    dev = torch.device("cuda")
    torch.set_num_threads(max(1, torch.get_num_threads()))
    model, cfg = bench.build_model("1.3b", dev)
    ref = copy.deepcopy(model).to("cpu")
    _fp32_head(model)
    _fp32_head(ref)
    mask = bench.MASK
    SL.patch_model_with_sabrecoder_attention(model, None, topk_blocks=0, verbose=False, **mask)
    ids, spans = bench.prompt_inputs(PROMPT, 1000, cfg.vocab_size)
    mb = StructureAwareMaskBuilder(None, **mask)
    bi, bc, bm = mb.build_block_indices_from_spans(spans, dev)
    patch_oracle(ref, bi.cpu(), bc.cpu(), mask["block_size"])
    ids_t = torch.from_numpy(ids)

    SL.set_current_code("<synthetic prompt>")
    SL.set_precomputed_blocks(bi, bc)
    ours, ours_logits = [], []
    try:
        with torch.no_grad():
            cache = SabreKVCache(cfg, batch_size=1, max_cache_len=PROMPT + STEPS + 64, device=dev)
            logits = model(input_ids=ids_t.to(dev), past_key_values=cache, use_cache=True,
                           logits_to_keep=1).logits
            for _ in range(STEPS):
                lg = logits[0, -1].float()
                tok = int(lg.argmax())
                ours.append(tok)
                ours_logits.append(lg.cpu())
                logits = model(input_ids=torch.tensor([[tok]], device=dev), past_key_values=cache,
                               use_cache=True).logits
    finally:
        SL.clear_current_code()
        SL.clear_precomputed_blocks()
    del model
    torch.cuda.empty_cache()

    def teacher_forced(m):
        """Logits (fp32, [steps, vocab]) of model m over the prompt and our tokens."""
        out = []
        with torch.no_grad():
            cc = DynamicCache()
            lb = m(input_ids=ids_t, past_key_values=cc, use_cache=True, logits_to_keep=1).logits
            for tok in ours:
                out.append(lb[0, -1].float())
                lb = m(input_ids=torch.tensor([[tok]]), past_key_values=cc, use_cache=True).logits
        return torch.stack(out)

    ref16 = teacher_forced(ref)
    ref.float()
    ref32 = teacher_forced(ref)
    a = torch.stack(ours_logits)
    err_ours = (a - ref32).abs().amax(-1)
    err_ref = (ref16 - ref32).abs().amax(-1)
    bound = NOISE_FACTOR * err_ref.max().item()
    top2 = ref32.topk(2, dim=-1)
    margin = (top2.values[:, 0] - top2.values[:, 1])
    exact = top2.indices[:, 0]
    toks = torch.tensor(ours)
    gap = top2.values[:, 0] - ref32.gather(1, toks[:, None])[:, 0]
    differ = [i for i in range(STEPS) if int(toks[i]) != int(exact[i])]
    ref_differ = [i for i in range(STEPS) if int(ref16[i].argmax()) != int(exact[i])]
    first = differ[0] if differ else None
    report = (f"tokens {ours}; steps where ours differs from the exact greedy choice: {differ} "
              f"(first: {'none' if first is None else f'step {first}, ours {ours[first]}, exact {int(exact[first])}, exact top-2 margin {margin[first]:.4f}, exact gap to ours {gap[first]:.4f}'}); "
              f"the reference's own bf16 run differs at {ref_differ}; exact top-2 margins min {margin.min():.4f} / "
              f"median {margin.median():.4f}; logit error ours max {err_ours.max():.4f} / median "
              f"{err_ours.median():.4f}, reference bf16 max {err_ref.max():.4f} / median {err_ref.median():.4f}; "
              f"bound {bound:.4f}")
    print(report)
    assert (err_ours <= bound).all(), report
    assert all(gap[i].item() <= bound for i in differ), report
    assert len(differ) <= STEPS // 4, report
