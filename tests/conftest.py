import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

from llm_embed_b200 import synth  # noqa: E402
from helpers import MODEL_DIR  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU; run with -m gpu")


@pytest.fixture(scope="session")
def model_path():
    """Factory: path of a cached synthetic model for a spec or config name."""
    def get(spec_or_name):
        return synth.cached_model(spec_or_name, MODEL_DIR)
    return get
