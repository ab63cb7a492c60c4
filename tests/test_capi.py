"""The C-ABI library on the CPU: it loads, exports every symbol the header
declares, and the binding is generated from that header.  No compute calls."""
import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest

from gollama_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent
HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared(path: Path) -> list[str]:
    text = re.sub(r"/\*.*?\*/", " ", path.read_text(), flags=re.S)
    return re.findall(r"GLC_API\s+int\s+(glc_\w+)\s*\(", text)


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    names = [n for h in HEADERS for n in declared(h)]
    assert len(names) >= 50
    for n in names:
        assert hasattr(lib, n), n
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (glc_\w+)", out))
    assert set(names) == exported, set(names) ^ exported


def test_binding_covers_header():
    assert set(_lib.SIGNATURES) == {n for h in HEADERS for n in declared(h)}


def test_every_entry_point_cites_the_reference_or_says_it_has_none():
    """Each declaration's comment (the block above it, or above the group of
    declarations and #defines it belongs to) cites the reference function it
    replaces by Go file, or says it has no reference counterpart."""
    uncited = []
    for h in HEADERS:
        lines = h.read_text().split("\n")
        for i, line in enumerate(lines):
            if not line.startswith("GLC_API"):
                continue
            j = i - 1
            while j >= 0 and (lines[j].startswith(("GLC_API", "#define")) or
                              (lines[j].startswith(" ") and not lines[j].lstrip().startswith("*"))):
                j -= 1
            block = []
            while j >= 0 and (lines[j].lstrip().startswith(("/*", "*", "//")) or lines[j].rstrip().endswith("*/")):
                block.append(lines[j])
                j -= 1
            if not re.search(r"\.go\b|counterpart", " ".join(block)):
                uncited.append(re.search(r"(glc_\w+)\s*\(", line).group(1))
    assert not uncited, uncited


def test_config_struct_layout_matches_header():
    lib = _lib.load()
    cfg = _lib.TrainConfigC()
    assert lib.glc_default_train_config(C.byref(cfg)) == 0
    # DefaultTrainConfig (pkg/train/trainer.go:43-69) and NewAdamW (optimizer.go:24-34)
    assert (cfg.vocab_size, cfg.hidden_size, cfg.num_layers, cfg.num_heads) == (32000, 512, 8, 8)
    assert (cfg.intermediate_size, cfg.max_seq_len, cfg.batch_size, cfg.block_size) == (1408, 512, 4, 256)
    assert (cfg.warmup_steps, cfg.max_steps) == (100, 10000)
    assert abs(cfg.learning_rate - 3e-4) < 1e-10 and abs(cfg.weight_decay - 0.01) < 1e-9
    assert abs(cfg.beta2 - 0.999) < 1e-7 and abs(cfg.epsilon - 1e-8) < 1e-15
    assert cfg.world_size == 1 and cfg.seed == 42


def test_invalid_arguments_fail_without_a_device():
    lib = _lib.load()
    assert lib.glc_init(0, None) == -1
    assert lib.glc_rope_table(3, 4, C.c_float(10000.0), None, None) == -1
    assert lib.glc_default_train_config(None) == -1


def test_rope_table_host():
    import numpy as np

    lib = _lib.load()
    c = np.zeros((8, 4), np.float32)
    s = np.zeros((8, 4), np.float32)
    assert lib.glc_rope_table(8, 8, C.c_float(10000.0), c.ctypes.data_as(C.c_void_p), s.ctypes.data_as(C.c_void_p)) == 0
    pos = np.arange(8)[:, None]
    freq = 1.0 / 10000.0 ** (2 * np.arange(4) / 8)
    assert np.array_equal(c, np.cos(pos * freq).astype(np.float32))
    assert np.array_equal(s, np.sin(pos * freq).astype(np.float32))


def test_no_cpu_fallback_without_gpu():
    """Without an sm_100 device the context cannot open: no CPU path exists."""
    from gollama_b200.device import Context, GlcError

    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(GlcError):
        Context(0)
