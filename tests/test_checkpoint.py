"""Checkpoint files (host side, no GPU).

Trainer.SaveCheckpoint (pkg/train/trainer.go:554-584) prints a header, then
every parameter value with fmt's `%v` and a trailing space, one line per
parameter.  The library's writer is compared byte for byte with an
independent formatter here: numpy's shortest round-trip digits for float32
(Dragon4, np.format_float_scientific(unique=True)) laid out by Go's rules for
the shortest `%g` (strconv/ftoa.go: scientific when the decimal exponent is
< -4 or >= 6, exponent with a sign and at least two digits; positional
otherwise; "+Inf", "-Inf", "NaN", "-0").  The reader must accept that text
and return the same float32 bits; the binary state file must round-trip and
refuse corrupt, truncated and mismatched files."""
import ctypes as C
import math
import struct

import numpy as np
import pytest

from gollama_b200 import _lib
from gollama_b200 import checkpoint as ck
from gollama_b200.device import GlcError
from gollama_b200.train import SEMANTICS_LLAMA, TrainConfig

GLC_ERR_INVALID, GLC_ERR_IO = -1, -7

REF_CFG = TrainConfig(VocabSize=64, HiddenSize=16, NumLayers=2, NumHeads=2, IntermediateSize=32, MaxSeqLen=8)
LLAMA_CFG = TrainConfig(VocabSize=96, HiddenSize=32, NumLayers=1, NumHeads=4, NumKVHeads=2, IntermediateSize=48,
                        MaxSeqLen=16, Semantics=SEMANTICS_LLAMA)


def go_v(x) -> str:
    """fmt.Sprintf("%v", float32(x)) following strconv.FormatFloat(v, 'g', -1, 32)."""
    x = np.float32(x)
    if np.isnan(x):
        return "NaN"
    if np.isinf(x):
        return "+Inf" if x > 0 else "-Inf"
    neg = bool(np.signbit(x))
    if x == 0:
        return "-0" if neg else "0"
    sci = np.format_float_scientific(abs(x), unique=True, trim="-")
    mant, exp = sci.split("e")
    digits = mant.replace(".", "")
    e = int(exp)
    if e < -4 or e >= 6:
        body = digits[0] + ("." + digits[1:] if len(digits) > 1 else "")
        body += "e" + ("-" if e < 0 else "+") + f"{abs(e):02d}"
    else:
        dp = e + 1
        whole = digits[:dp].ljust(dp, "0") if dp > 0 else "0"
        frac = ("0" * -dp + digits) if dp <= 0 else digits[dp:]
        body = whole + ("." + frac if frac else "")
    return ("-" if neg else "") + body


def sizes(cfg):
    plan_n = C.c_int()
    c = cfg.to_c()
    lib = _lib.load()
    assert lib.glc_dp_bucket_plan(C.byref(c), None, None, 0, C.byref(plan_n)) == 0
    d, F, V = cfg.HiddenSize, cfg.IntermediateSize, cfg.VocabSize
    kvd = (cfg.NumKVHeads or cfg.NumHeads) * (d // cfg.NumHeads) if cfg.Semantics == SEMANTICS_LLAMA else d
    out = [V * d] + ([] if cfg.Semantics == SEMANTICS_LLAMA else [cfg.MaxSeqLen * d])
    for _ in range(cfg.NumLayers):
        out += [d, d * d, kvd * d, kvd * d, d * d, d, F * d, F * d, d * F]
    return out + [d]


def expected_text(cfg, step, flat) -> bytes:
    lines = ["GOLLAMA_CKPT", f"step={step}", f"vocab_size={cfg.VocabSize}", f"hidden_size={cfg.HiddenSize}",
             f"num_layers={cfg.NumLayers}", f"num_heads={cfg.NumHeads}", f"intermediate_size={cfg.IntermediateSize}",
             "WEIGHTS"]
    out = "\n".join(lines) + "\n"
    off = 0
    for n in sizes(cfg):
        out += "".join(go_v(v) + " " for v in flat[off : off + n]) + "\n"
        off += n
    return out.encode()


# fmt %v outputs of float32 values, by Go's documented rules
KNOWN = [
    (0.1, "0.1"), (0.02, "0.02"), (1.0, "1"), (-2.5, "-2.5"), (100000.0, "100000"), (123456.7, "123456.7"),
    (1e6, "1e+06"), (1.5e6, "1.5e+06"), (16777216.0, "1.6777216e+07"), (0.0001, "0.0001"), (0.00012, "0.00012"),
    (1e-5, "1e-05"), (1.5e-5, "1.5e-05"), (1.0 / 3.0, "0.33333334"), (3.4028235e38, "3.4028235e+38"),
    (1e-45, "1e-45"), (1.1754944e-38, "1.1754944e-38"), (0.0, "0"), (-0.0, "-0"), (math.inf, "+Inf"),
    (-math.inf, "-Inf"), (math.nan, "NaN"), (999999.94, "999999.94"), (9.999999e-5, "9.999999e-05"),
]


@pytest.mark.parametrize("value,text", KNOWN, ids=[t for _, t in KNOWN])
def test_go_formatter_known_values(value, text):
    assert go_v(value) == text


def special_params(n, seed):
    rng = np.random.default_rng(seed)
    flat = (rng.standard_normal(n) * 0.02).astype(np.float32)
    vals = np.array([v for v, _ in KNOWN], np.float32)
    flat[: len(vals)] = vals
    # random bit patterns: every exponent, subnormals, large and tiny magnitudes
    bits = rng.integers(0, 2**32, size=n // 3, dtype=np.uint64).astype(np.uint32)
    pos = rng.choice(np.arange(len(vals), n), size=bits.size, replace=False)
    flat[pos] = bits.view(np.float32)
    return flat


@pytest.mark.parametrize("cfg", [REF_CFG, LLAMA_CFG], ids=["reference", "llama"])
def test_text_checkpoint_bytes_and_round_trip(tmp_path, cfg):
    n = ck.param_count(cfg)
    assert n == sum(sizes(cfg))
    flat = special_params(n, 3)
    path = tmp_path / "checkpoint_12.bin"
    ck.write_checkpoint(path, 12, cfg, flat)
    got = path.read_bytes()
    want = expected_text(cfg, 12, flat)
    if got != want:
        a, b = got.split(b" "), want.split(b" ")
        first = next(i for i, (x, y) in enumerate(zip(a, b)) if x != y)
        pytest.fail(f"first differing token {first}: library {a[first]!r}, Go rules {b[first]!r}")
    step, back = ck.read_checkpoint(path, cfg)
    assert step == 12
    nan = np.isnan(flat)
    assert np.array_equal(np.isnan(back), nan)
    assert np.array_equal(back[~nan].view(np.uint32), flat[~nan].view(np.uint32))


def test_reader_accepts_text_written_by_go_rules(tmp_path):
    """A file produced by the formatter above (what the reference writes) reads
    back bit for bit, independent of the library's writer."""
    n = ck.param_count(REF_CFG)
    flat = special_params(n, 9)
    path = tmp_path / "checkpoint_3.bin"
    path.write_bytes(expected_text(REF_CFG, 3, flat))
    step, back = ck.read_checkpoint(path, REF_CFG)
    assert step == 3
    nan = np.isnan(flat)
    assert np.array_equal(back[~nan].view(np.uint32), flat[~nan].view(np.uint32))


def _err(fn, *args):
    with pytest.raises(GlcError) as e:
        fn(*args)
    return e.value


def test_text_reader_refuses_bad_files(tmp_path):
    n = ck.param_count(REF_CFG)
    flat = (np.arange(n, dtype=np.float32) - 100) / 7
    good = expected_text(REF_CFG, 5, flat)
    path = tmp_path / "c.bin"

    def read(blob):
        path.write_bytes(blob)
        return _err(ck.read_checkpoint, path, REF_CFG)

    assert read(b"NOT_A_CKPT\n").code == GLC_ERR_IO
    assert read(good.replace(b"hidden_size=16", b"hidden_size=32")).code == GLC_ERR_INVALID
    assert "hidden_size" in str(read(good.replace(b"hidden_size=16", b"hidden_size=32")))
    assert read(good.replace(b"step=5", b"step=x")).code == GLC_ERR_IO
    assert read(good[: len(good) // 2]).code in (GLC_ERR_IO, GLC_ERR_INVALID)  # truncated
    lines = good.split(b"\n")
    short = lines[:8] + [lines[8].rsplit(b" ", 2)[0] + b" "] + lines[9:]  # one value fewer in parameter 0
    assert read(b"\n".join(short)).code == GLC_ERR_INVALID
    extra = lines[:8] + [lines[8] + b"1 "] + lines[9:]
    assert read(b"\n".join(extra)).code == GLC_ERR_INVALID
    assert read(good + b"0 \n").code == GLC_ERR_INVALID  # a parameter too many
    bad = lines[:8] + [lines[8].replace(b" ", b" 1x", 1)] + lines[9:]
    assert read(b"\n".join(bad)).code == GLC_ERR_IO
    for tok in (b"+1", b"Inf", b"nan", b"1e", b"", b"0x1p3"):  # never printed by %v
        toks = lines[8].split(b" ")
        toks[1] = tok
        assert read(b"\n".join(lines[:8] + [b" ".join(toks)] + lines[9:])).code in (GLC_ERR_IO, GLC_ERR_INVALID), tok
    assert _err(ck.read_checkpoint, tmp_path / "missing.bin", REF_CFG).code == GLC_ERR_IO
    # the reference writes into an existing directory only (trainer.go:558-562)
    assert _err(ck.write_checkpoint, tmp_path / "no_dir" / "c.bin", 1, REF_CFG, flat).code == GLC_ERR_IO
    assert _err(ck.write_checkpoint, path, 1, REF_CFG, flat[:-1]).code == GLC_ERR_INVALID


@pytest.mark.parametrize("cfg", [REF_CFG, LLAMA_CFG], ids=["reference", "llama"])
def test_state_round_trip(tmp_path, cfg):
    n = ck.param_count(cfg)
    rng = np.random.default_rng(4)
    p, m, v = (rng.standard_normal(n).astype(np.float32) for _ in range(3))
    path = tmp_path / "s.glcstate"
    ck.write_state(path, cfg, 17, 16, p, m, v)
    assert path.stat().st_size == 80 + 12 * n
    assert path.read_bytes()[:8] == b"GLCSTATE"
    step, adam_step, p2, m2, v2 = ck.read_state(path, cfg)
    assert (step, adam_step) == (17, 16)
    for a, b in ((p, p2), (m, m2), (v, v2)):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_state_refuses_corrupt_truncated_and_mismatched(tmp_path):
    n = ck.param_count(REF_CFG)
    rng = np.random.default_rng(5)
    p, m, v = (rng.standard_normal(n).astype(np.float32) for _ in range(3))
    path = tmp_path / "s.glcstate"
    ck.write_state(path, REF_CFG, 3, 3, p, m, v)
    blob = bytearray(path.read_bytes())
    out = np.full(n, 7, np.float32)

    def read(b, cfg=REF_CFG):
        path.write_bytes(bytes(b))
        return _err(ck.read_state, path, cfg)

    flipped = bytearray(blob)
    flipped[80 + 4 * n + 123] ^= 0x10  # one bit of m
    e = read(flipped)
    assert e.code == GLC_ERR_IO and "hash" in str(e)
    stepped = bytearray(blob)
    stepped[16] ^= 1  # the trainer step: covered by the hash too
    e = read(stepped)
    assert e.code == GLC_ERR_IO and "hash" in str(e)
    assert read(blob[:-4]).code == GLC_ERR_IO
    assert read(blob + b"\0\0\0\0").code == GLC_ERR_IO
    assert read(b"GLCSTATX" + blob[8:]).code == GLC_ERR_IO
    assert read(blob[:8] + struct.pack("<I", 2) + blob[12:]).code == GLC_ERR_IO
    other = TrainConfig(**{**REF_CFG.__dict__, "NumLayers": 3})
    assert read(blob, other).code == GLC_ERR_INVALID
    wider = TrainConfig(**{**REF_CFG.__dict__, "MaxSeqLen": 16})  # the text header omits it; the state does not
    assert "max_seq_len" in str(read(blob, wider))
    # nothing of a refused file reaches the caller's buffers
    path.write_bytes(bytes(flipped))
    step, adam = C.c_int(-1), C.c_int(-1)
    c = REF_CFG.to_c()
    rc = _lib.load().glc_state_read(str(path).encode(), C.byref(c), C.byref(step), C.byref(adam),
                                    out.ctypes.data_as(C.c_void_p), out.ctypes.data_as(C.c_void_p),
                                    out.ctypes.data_as(C.c_void_p), n)
    assert rc == GLC_ERR_IO and step.value == -1 and np.all(out == 7)


def test_last_error_without_context(tmp_path):
    lib = _lib.load()
    c = REF_CFG.to_c()
    step = C.c_int()
    buf = np.zeros(4, np.float32)
    rc = lib.glc_checkpoint_read(str(tmp_path / "none.bin").encode(), C.byref(c), C.byref(step),
                                 buf.ctypes.data_as(C.c_void_p), 4)
    assert rc == GLC_ERR_INVALID  # n is not the parameter count
    msg = C.create_string_buffer(256)
    assert lib.glc_last_error(None, msg, 256) == 0
    assert b"parameter count" in msg.value


def test_text_checkpoint_across_blocks_and_threads(tmp_path):
    """A file larger than the reader's 64 MiB block: values and line ends cut
    across blocks and per-thread slices read back bit for bit, and errors late
    in the file name the right parameter."""
    cfg = TrainConfig(VocabSize=32000, HiddenSize=192, NumLayers=1, NumHeads=2, IntermediateSize=512, MaxSeqLen=64)
    n = ck.param_count(cfg)
    flat = special_params(n, 11)
    path = tmp_path / "big.bin"
    ck.write_checkpoint(path, 40, cfg, flat)
    assert path.stat().st_size > (1 << 26)
    step, back = ck.read_checkpoint(path, cfg)
    assert step == 40
    nan = np.isnan(flat)
    assert np.array_equal(back[~nan].view(np.uint32), flat[~nan].view(np.uint32))

    blob = path.read_bytes()
    lines = blob.split(b"\n")
    # the last parameter (output norm) holds a malformed value
    last = lines[-2].split(b" ")
    last[5] = b"1.0.0"
    path.write_bytes(b"\n".join(lines[:-2] + [b" ".join(last)] + lines[-1:]))
    e = _err(ck.read_checkpoint, path, cfg)
    assert e.code == GLC_ERR_IO and f"in parameter {len(sizes(cfg)) - 1}" in str(e)
    # the embedding (first line, spanning blocks and slices) misses one value
    emb = lines[8].split(b" ")
    path.write_bytes(b"\n".join(lines[:8] + [b" ".join(emb[:1000] + emb[1001:])] + lines[9:]))
    e = _err(ck.read_checkpoint, path, cfg)
    assert e.code == GLC_ERR_INVALID and "parameter 0 holds" in str(e)
    # cut inside the second-to-last parameter
    path.write_bytes(blob[: len(blob) - len(lines[-2]) - 1000])
    e = _err(ck.read_checkpoint, path, cfg)
    assert e.code == GLC_ERR_IO


def test_text_reader_survives_random_mutations(tmp_path):
    """Random byte mutations of a valid file end in an error status or, when
    the mutated text is still a well-formed checkpoint of the model (the
    reader takes any plain decimal spelling, not only %v's), in the values its
    tokens spell; never a crash."""
    n = ck.param_count(REF_CFG)
    flat = (np.random.default_rng(12).standard_normal(n) * 0.02).astype(np.float32)
    good = bytearray(expected_text(REF_CFG, 9, flat))
    rng = np.random.default_rng(13)
    path = tmp_path / "m.bin"
    alphabet = b"0123456789.-+e \nNaInf"
    accepted = 0
    for _ in range(300):
        b = bytearray(good)
        for _ in range(int(rng.integers(1, 4))):
            pos = int(rng.integers(0, len(b)))
            op = rng.integers(0, 3)
            if op == 0:
                b[pos] = alphabet[int(rng.integers(0, len(alphabet)))]
            elif op == 1:
                del b[pos]
            else:
                b.insert(pos, alphabet[int(rng.integers(0, len(alphabet)))])
        path.write_bytes(bytes(b))
        try:
            step, back = ck.read_checkpoint(path, REF_CFG)
        except GlcError as e:
            assert e.code in (GLC_ERR_IO, GLC_ERR_INVALID)
            continue
        accepted += 1
        # every value is its token's float32 (Python parses through float64,
        # which may round twice: within one float32 ulp)
        toks = [t for line in bytes(b).split(b"\n")[8:] for t in line.split(b" ") if t]
        assert len(toks) == n
        ref = np.array([float(t.decode()) for t in toks], np.float64).astype(np.float32)
        fin = np.isfinite(ref)
        assert np.array_equal(np.isnan(back), np.isnan(ref))
        diff = np.abs(back[fin].view(np.int32).astype(np.int64) - ref[fin].view(np.int32).astype(np.int64))
        assert diff.max(initial=0) <= 1
    assert accepted < 300  # most mutations are refused
