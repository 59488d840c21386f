"""The verifier stage against Hugging Face's own Qwen3.5 implementation (CPU).

The same synthetic HF-layout checkpoint (three gated-delta-net layers and one
gated full-attention layer, bf16 weights) is loaded into our ``QwenStage`` and
into ``transformers``' ``Qwen3_5ForCausalLM`` (fp32, torch fallback kernels).
The captured decoder outputs and the final normed hidden state must agree to bf16
resolution. This is the role of the reference's HF oracle (experiments/compare.py:
138-181), run here on the CPU instead of an inference GPU.
"""

import json

import pytest
import torch

from nanospec_b200.models import verifier as V

transformers = pytest.importorskip("transformers")


def _hf_model(tc, state):
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5ForCausalLM

    cfg = Qwen3_5TextConfig(**tc, tie_word_embeddings=False)
    cfg._attn_implementation = "eager"
    model = Qwen3_5ForCausalLM(cfg).float().eval()
    prefix = "model.language_model."
    renamed = {("model." + k[len(prefix):] if k.startswith(prefix) else k): v.float() for k, v in state.items()}
    missing, unexpected = model.load_state_dict(renamed, strict=False)
    assert not missing and not unexpected, (missing, unexpected)
    return model


def _close(a, b, rel_tol):
    a, b = a.float(), b.float()
    cos = torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0).item()
    rel = ((a - b).norm() / b.norm()).item()
    assert cos > 0.9995 and rel < rel_tol, (cos, rel)


def test_stage_matches_hf_qwen3_5(tmp_path):
    from safetensors.torch import load_file

    tc = V.tiny_hybrid_text_config()
    V.write_synthetic_checkpoint(tmp_path, tc, seed=3, fp8=False, dtype=torch.bfloat16)
    state = {}
    index = json.loads((tmp_path / "model.safetensors.index.json").read_text())["weight_map"]
    for name in sorted(set(index.values())):
        state.update(load_file(str(tmp_path / name)))
    model = _hf_model(tc, state)
    ids = torch.randint(0, tc["vocab_size"], (2, 40), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        ref = model.model(input_ids=ids, output_hidden_states=True)
    stage = V.QwenStage(V.Checkpoint(tmp_path), 0, tc["num_hidden_layers"], device=torch.device("cpu"),
                        first=True, last=True)
    final, captured = V.stage_forward(stage, ids, capture=(0, 1, 2))
    for li in (0, 1, 2):  # gated delta net layers
        _close(captured[li], ref.hidden_states[li + 1], 1e-2)
    _close(final, ref.last_hidden_state, 1.5e-2)  # after the full-attention layer and the final norm
