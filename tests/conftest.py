"""Shared test set-up: the `gpu` marker, the package loader and the synthetic weights."""
from __future__ import annotations

import importlib.util
import json
import os
import sys
import tempfile
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG_DIR = ROOT / "dsh-moss-tts_b200"
sys.path.insert(0, str(ROOT / "oracle"))
sys.path.insert(0, str(ROOT / "tests"))


def load_package():
    """Import the package directory (its name is not a Python identifier) as `moss_b200`."""
    if "moss_b200" in sys.modules:
        return sys.modules["moss_b200"]
    spec = importlib.util.spec_from_file_location("moss_b200", PKG_DIR / "__init__.py",
                                                  submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["moss_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


load_package()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session")
def weights_path() -> str:
    """The seed-0 synthetic model (125,047,648 B), generated once per machine and checked
    against the digest recorded by tests/golden/make_golden.py."""
    from moss_b200 import mossfile
    meta = json.loads((ROOT / "tests" / "golden" / "weights.json").read_text())
    path = Path(os.environ.get("MOSS_TEST_WEIGHTS", Path(tempfile.gettempdir()) / "moss_b200_w0.moss"))
    mossfile.ensure_synth_weights(path, meta["seed"])
    return str(path)


@pytest.fixture(scope="session")
def weights_digest_ok(weights_path) -> bool:
    import hashlib
    meta = json.loads((ROOT / "tests" / "golden" / "weights.json").read_text())
    h = hashlib.sha256(Path(weights_path).read_bytes()).hexdigest()
    return h == meta["sha256"]


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return ROOT / "tests" / "golden"


@pytest.fixture(scope="session")
def decoder_file() -> str:
    """The seed-1 synthetic audio codec decoder, generated once per machine (about a second)."""
    from golden_inputs import CODEC_DECODER_SEED
    from moss_b200 import codecfile
    path = Path(tempfile.gettempdir()) / f"moss_b200_dec{CODEC_DECODER_SEED}.moss"
    return codecfile.ensure_synth_decoder(path, CODEC_DECODER_SEED)
