"""Shared helpers for the test suite."""
import os

from llm_embed_b200 import synth

MODEL_DIR = os.environ.get("LLMEMBED_MODEL_DIR", "/tmp/llm_embed_b200_models")


def small_spec(weight_type=synth.GGML_Q8_0, embd_type=synth.GGML_Q8_0, layers=2, vocab=2048, seed=11, context=2048):
    """A 2-layer, full-width nomic-bert spec with a small vocabulary."""
    return synth.ModelSpec(layers=layers, vocab=vocab, seed=seed, context=context, embd_type=embd_type,
                           weight_types=(weight_type,) * 5)
