"""HF transformers Mamba-1 through patch() on the GPU (reference
tests/check_hf_patch.py, without downloaded weights: a random-init model).

The patched slow_forward must reproduce the unpatched one (logits within
1e-4 relative), engage the kernel on every layer, seed the caches so greedy
generation continues identically, and unpatch() must restore the original."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def tiny_model(layers=3):
    from transformers import MambaConfig, MambaForCausalLM
    cfg = MambaConfig(vocab_size=500, hidden_size=64, state_size=16, num_hidden_layers=layers,
                      expand=2, conv_kernel=4, time_step_rank=8, use_cache=True)
    torch.manual_seed(0)
    return MambaForCausalLM(cfg).cuda().eval()


def test_patched_logits_and_generation_match_unpatched():
    import armhackathon_b200 as arm
    model = tiny_model()
    ids = torch.randint(0, 500, (2, 77), device="cuda")
    with torch.no_grad():
        want = model(ids).logits
        want_gen = model.generate(ids[:1, :20], max_new_tokens=8, do_sample=False)
    targets = arm.patch()
    try:
        assert targets
        before = arm.stats()["fast_calls"]
        dec_before = arm.stats()["decode_calls"]
        with torch.no_grad():
            got = model(ids).logits
            got_gen = model.generate(ids[:1, :20], max_new_tokens=8, do_sample=False)
        assert arm.stats()["fast_calls"] - before >= 3 * 2  # every layer, both calls
        # generate's 7 single-token steps run through selective_state_update
        assert arm.stats()["decode_calls"] - dec_before == 3 * 7
        rel = (got - want).abs().max() / want.abs().max()
        assert rel < 1e-4, rel
        assert torch.equal(got_gen, want_gen)
    finally:
        assert arm.unpatch()
    from transformers.models.mamba import modeling_mamba
    assert not getattr(modeling_mamba.MambaMixer.slow_forward, "__name__", "") == "slow_forward" \
        or modeling_mamba.MambaMixer.slow_forward.__qualname__.startswith("MambaMixer")
