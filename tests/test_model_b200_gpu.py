"""The B200 backend against the eager oracle on identical bf16 weights."""

from __future__ import annotations

import pytest
import torch

from cs244c_llama_zero_b200.models import LlamaForCausalLM, ModelConfig

pytestmark = pytest.mark.gpu


def _cfg(hd: int = 64, tied: bool = True) -> ModelConfig:
    return ModelConfig(name="b200_test", vocab_size=1024, max_seq_len=256, dim=4 * hd, n_layers=2, n_heads=4,
                       n_kv_heads=2, ffn_dim=512, rope_theta=10000.0, tie_word_embeddings=tied)


def _pair(cfg):
    torch.manual_seed(0)
    ref = LlamaForCausalLM(cfg).cuda().to(torch.bfloat16)
    fast = LlamaForCausalLM(cfg).cuda().to(torch.bfloat16)
    fast.load_state_dict(ref.state_dict())
    fast.set_backend("b200")
    return ref, fast


@pytest.mark.parametrize("hd,tied", [(64, True), (128, False)])
def test_b200_loss_and_grads_match_eager(hd, tied):
    """The fp32 eager model is the oracle; the B200 path must be as close to it as eager bf16 is."""
    cfg = _cfg(hd, tied)
    ref, fast = _pair(cfg)
    oracle = LlamaForCausalLM(cfg).cuda()
    oracle.load_state_dict({k: v.float() for k, v in ref.state_dict().items()})
    ids = torch.randint(0, cfg.vocab_size, (2, cfg.max_seq_len), device="cuda")
    l_oracle = oracle(input_ids=ids, labels=ids, return_logits=False).loss
    with torch.autocast("cuda", dtype=torch.bfloat16):
        l_ref = ref(input_ids=ids, labels=ids, return_logits=False).loss
        l_fast = fast(input_ids=ids, labels=ids, return_logits=False).loss
    torch.testing.assert_close(l_fast.float(), l_oracle, rtol=1e-2, atol=1e-2)
    l_oracle.backward()
    l_ref.backward()
    l_fast.backward()
    for (name, po), (_, pr), (_, pf) in zip(oracle.named_parameters(), ref.named_parameters(), fast.named_parameters()):
        go = po.grad
        err_fast = (pf.grad.float() - go).norm().item()
        err_eager = (pr.grad.float() - go).norm().item()
        scale = go.norm().item() + 1e-12
        assert err_fast <= 2.0 * err_eager + 0.02 * scale, (
            f"{name}: b200 err {err_fast:.3g}, eager-bf16 err {err_eager:.3g}, grad norm {scale:.3g}")


def test_b200_engine_trains(tmp_path):
    from cs244c_llama_zero_b200.parallel.zero import ZeROStage0DDP

    cfg = _cfg(64)
    _, model = _pair(cfg)
    engine = ZeROStage0DDP(model=model, lr=3e-3, weight_decay=0.0)
    ids = torch.randint(0, cfg.vocab_size, (4, cfg.max_seq_len), device="cuda")
    losses = []
    for _ in range(15):
        engine.zero_grad()
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = model(input_ids=ids, labels=ids, return_logits=False).loss
        engine.backward(loss)
        engine.step()
        losses.append(float(loss))
    assert losses[-1] < 0.8 * losses[0], losses
