"""The model loader's host side without a GPU: the GGUF reader (trochilus_b200/csrc/gguf_file.h) against gguf-py's
own reader on files gguf-py wrote (every tensor's type, dimensions, offset and size), its refusal of malformed files
in a child process (truncations and corrupted bytes end in an error, never a crash), and
tr_gpu_moe_config_from_gguf's configuration and messages on the reference's names and checks
(src/models/olmoe.c:541-641, 895-906)."""
import os
import subprocess

import numpy as np
import pytest

from tests.gguf_fixture import write_olmoe_moe
from trochilus_b200 import gguf_blocks as gb

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
E, H, F = 8, 512, 256


@pytest.fixture(scope="module")
def dump(tmp_path_factory):
    exe = str(tmp_path_factory.mktemp("gguf") / "gguf_dump")
    # with the address and undefined-behaviour sanitizers: a read outside the mapping ends the program with an error
    subprocess.check_call(["g++", "-O1", "-g", "-std=c++17", "-Wall", "-Werror", "-fsanitize=address,undefined",
                           "-fno-sanitize-recover=all", os.path.join(ROOT, "tests", "gguf_dump.cpp"), "-o", exe])
    return exe


def _layers(router_type=gb.F32, n=2, gate=gb.Q8_0, down=gb.Q6_K):
    return [gb.make_layer(40 + i, E, H, F, gate, down, router_type) for i in range(n)]


def _norms(n=2):
    return [np.linspace(0.5 + i, 1.5, H).astype(np.float32) for i in range(n)]


def test_reader_matches_gguf_py(tmp_path, dump):
    import gguf
    p = write_olmoe_moe(tmp_path / "m.gguf", _layers(), _norms())
    r = gguf.GGUFReader(str(p))
    names = [t.name for t in r.tensors]
    out = subprocess.run([dump, str(p), *names, "blk.9.ffn_norm.weight"], capture_output=True, text=True, check=True)
    lines = out.stdout.splitlines()
    assert lines[0] == "ok 3" and "absent blk.9.ffn_norm.weight" in lines and f"expert_count {E}" in lines
    got = {ln.split()[1]: ln.split()[2:] for ln in lines if ln.startswith("tensor ")}
    assert len(got) == len(names) == 2 * 5
    for t in r.tensors:
        f = got[t.name]
        n_dims = int(f[1])
        assert int(f[0]) == int(t.tensor_type), t.name
        assert [int(v) for v in f[2:2 + n_dims]] == [int(v) for v in t.shape], t.name
        assert int(f[3 + n_dims]) == int(t.data_offset) and int(f[4 + n_dims]) == int(t.n_bytes), t.name


def test_malformed_files_end_in_errors(tmp_path, dump):
    p = write_olmoe_moe(tmp_path / "m.gguf", _layers(n=1), _norms(1))
    raw = open(p, "rb").read()
    header_end = raw.index(b"blk.0.ffn_down_exps.weight") + 64  # past the last directory entry
    rng = np.random.default_rng(0)
    cases = [raw[:n] for n in (0, 3, 8, 20, 100, header_end - 40, header_end, len(raw) // 2, len(raw) - 1)]
    for _ in range(300):  # corrupted bytes in the header and directory
        b = bytearray(raw)
        for _ in range(int(rng.integers(1, 4))):
            b[int(rng.integers(0, header_end))] = int(rng.integers(0, 256))
        cases.append(bytes(b))
    cases.append(b"GGUF" + (1).to_bytes(4, "little") + raw[8:])  # version 1
    q = tmp_path / "bad.gguf"
    errors = 0
    env = dict(os.environ, ASAN_OPTIONS="exitcode=86", UBSAN_OPTIONS="halt_on_error=1:exitcode=86")
    for c in cases:
        q.write_bytes(c)
        out = subprocess.run([dump, str(q)], capture_output=True, env=env)
        # 0 or 1 (an error message): never a signal or a sanitizer's report
        assert out.returncode in (0, 1), (out.returncode, out.stdout[:200], out.stderr[:400])
        errors += out.returncode == 1
    assert errors >= 10  # every truncation and the version among them


def test_config_from_gguf(tmp_path):
    from trochilus_b200 import moe
    p = write_olmoe_moe(tmp_path / "a.gguf", _layers(), _norms(), eps=2e-6, n_used=3, norm_topk=True)
    cfg, eps = moe.config_from_gguf(str(p), max_tokens=7)
    assert (cfg.n_layers, cfg.n_expert, cfg.n_used, cfg.n_embd, cfg.n_ff, cfg.norm_topk) == (2, E, 3, H, F, 1)
    assert (cfg.router_type, cfg.gate_type, cfg.down_type, cfg.max_tokens) == (gb.F32, gb.Q8_0, gb.Q6_K, 7)
    assert eps == np.float32(2e-6)
    # an F32 router whose values are all bfloat16 is taken as BF16 (olmoe.c:391), as is a BF16 one
    lays = _layers()
    for lay in lays:
        lay["router"] = gb.quantize(gb.F32, gb.round_to_bf16(lay["router"].view(np.float32).reshape(E, H)))
    cfg, _ = moe.config_from_gguf(str(write_olmoe_moe(tmp_path / "b.gguf", lays, _norms())))
    assert cfg.router_type == gb.BF16
    cfg, _ = moe.config_from_gguf(str(write_olmoe_moe(tmp_path / "c.gguf", _layers(gb.BF16), _norms(),
                                                      router_type=gb.BF16)))
    assert cfg.router_type == gb.BF16


@pytest.mark.parametrize("kind,match", [
    ("skip", "missing tensor 'blk.1.ffn_up_exps.weight'"),
    ("shape", r"tensor 'blk.0.ffn_down_exps.weight' has shape \[256, 1024, 4\], expected \[256, 512, 8\]"),
    ("arch", "general.architecture is 'llama'"),
    ("types", "layer 1's expert types differ"),
    ("key", "missing metadata key 'olmoe.expert_count'"),
    ("magic", "not a GGUF file"),
    ("nofile", "cannot open"),
])
def test_config_refusals(tmp_path, kind, match):
    from trochilus_b200 import moe
    p = tmp_path / "r.gguf"
    if kind == "skip":
        write_olmoe_moe(p, _layers(), _norms(), skip=("blk.1.ffn_up_exps.weight",))
    elif kind == "shape":
        write_olmoe_moe(p, _layers(), _norms(), reshape={"blk.0.ffn_down_exps.weight": (4, 1024, -1)})
    elif kind == "arch":
        write_olmoe_moe(p, _layers(), _norms(), arch="llama")
    elif kind == "types":  # layer 1's down Q8_0 while layer 0's is Q6_K
        lays = [_layers(n=1)[0], gb.make_layer(50, E, H, F, gb.Q8_0, gb.Q8_0, gb.F32)]
        write_olmoe_moe(p, lays, _norms(), down_types=[gb.Q6_K, gb.Q8_0])
    elif kind == "key":
        write_olmoe_moe(p, _layers(), _norms())
        raw = open(p, "rb").read().replace(b"olmoe.expert_count", b"olmoe.expert_cnt__")
        p.write_bytes(raw)
    elif kind == "magic":
        write_olmoe_moe(p, _layers(), _norms())
        p.write_bytes(b"GGUX" + open(p, "rb").read()[4:])
    with pytest.raises(RuntimeError, match=match):
        moe.config_from_gguf(str(p))
