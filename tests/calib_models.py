"""Tiny random-weight Hugging Face checkpoints for calibration-driver tests.

Written to a temporary directory (config, safetensors, a word-level tokenizer)
so the driver loads them through the same from_pretrained calls it uses for a
real checkpoint; no network and no downloaded weights are involved.
"""

from __future__ import annotations

import re
from pathlib import Path

import torch


def make_checkpoint(path: Path, model_type: str = "qwen2", seed: int = 0) -> Path:
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast

    from vllm_ascend_kvcompress.calibration import _BUILTIN_SECTIONS

    path.mkdir(parents=True, exist_ok=True)
    words = sorted(set(re.findall(r"\w+|[^\w\s]", " ".join(_BUILTIN_SECTIONS))))
    vocab = {"[UNK]": 0, "[BOS]": 1, **{w: i + 2 for i, w in enumerate(words)}}
    tok = Tokenizer(models.WordLevel(vocab, unk_token="[UNK]"))
    tok.pre_tokenizer = pre_tokenizers.Whitespace()
    PreTrainedTokenizerFast(tokenizer_object=tok, unk_token="[UNK]", bos_token="[BOS]",
                            model_max_length=8192).save_pretrained(path)
    torch.manual_seed(seed)
    common = dict(vocab_size=len(vocab), hidden_size=128, intermediate_size=256, num_hidden_layers=3,
                  num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=8192, rope_theta=1e6)
    if model_type == "qwen2":
        from transformers import Qwen2Config, Qwen2Model

        model = Qwen2Model(Qwen2Config(**common))
    elif model_type == "qwen3":
        from transformers import Qwen3Config, Qwen3Model

        model = Qwen3Model(Qwen3Config(head_dim=64, **common))
    else:
        raise ValueError(model_type)
    model.to(torch.bfloat16).save_pretrained(path)
    return path
