"""Our Qwen3 / Qwen3-MoE modules against Hugging Face transformers (CPU, fp32)."""
import pytest
import torch


@pytest.mark.parametrize("name", ["tiny-qwen3", "tiny-qwen3-moe"])
def test_matches_hf_loss_and_grads(tmp_path, name):
    transformers = pytest.importorskip("transformers")
    from parallel_b200.models.config import resolve_config
    from parallel_b200.models.qwen3 import build_model

    cfg = resolve_config(name)
    m = build_model(cfg, dtype=torch.float32, seed=0)
    cfg.save_pretrained(str(tmp_path))
    hc = transformers.AutoConfig.from_pretrained(str(tmp_path))
    hm = transformers.AutoModelForCausalLM.from_config(hc, attn_implementation="sdpa").float()
    res = hm.load_state_dict(m.state_dict(), strict=False)
    assert not res.missing_keys and not res.unexpected_keys
    ids = torch.randint(0, cfg.vocab_size, (2, 32), generator=torch.Generator().manual_seed(1))
    out = m(ids, labels=ids)            # HF convention: labels shifted inside the model
    ref = hm(input_ids=ids, labels=ids)
    torch.testing.assert_close(out.loss, ref.loss, rtol=1e-5, atol=1e-5)
    if cfg.is_moe:
        torch.testing.assert_close(out.aux_loss, ref.aux_loss, rtol=1e-5, atol=1e-6)
    out.loss.backward()
    ref.loss.backward()
    hp = dict(hm.named_parameters())
    for n, p in m.named_parameters():
        torch.testing.assert_close(p.grad, hp[n].grad, rtol=1e-4, atol=1e-6)


def test_double_shift_convention():
    """Non-model-parallel path: dataloader already shifted, model shifts again."""
    from parallel_b200.ops.functional import IGNORE_INDEX, shift_labels

    y = torch.tensor([[1, 2, 3, 4]])
    assert shift_labels(y).tolist() == [[2, 3, 4, IGNORE_INDEX]]
