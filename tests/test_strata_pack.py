"""The product .strata packer (sfk_strata_pack, `python -m
strataflow_b200.strata_pack`): the reference's pack_gguf_to_strata
(src/tws/strata_pack.cpp:251-1108) without LZ compression.  A GGUF written
from the CPU oracle's weights is packed and read back through the library's
own reader: every trunk tensor and every (layer, expert) bundle must be the
source's bytes, the superblock must carry the reference's v2 layout, and the
refusals of the reference's packer must hold (host-only, no GPU)."""
import struct
import zlib

import numpy as np
import pytest

from oracle import oracle as O
from strataflow_b200 import build as B
from strataflow_b200 import lib as L
from tests.strata_fixture import write_gguf


@pytest.fixture(scope="module", autouse=True)
def _lib():
    B.build()


def _cfg(**kw):
    d = dict(n_embd=256, n_head=8, n_head_kv=4, n_layer=2, n_ff=512, n_expert=8, n_expert_used=2, n_vocab=4096,
             n_ctx=80, rms_eps=1e-5, freq_base=10000.0, type_ffn_gu=O.Q4_K, type_ffn_down=O.Q6_K, type_attn=O.Q8_0)
    d.update(kw)
    return O.ModelConfig(**d)


@pytest.fixture(scope="module")
def model():
    cfg = _cfg()
    return cfg, O.Model(cfg, seed=33)


def _superblock(path):
    sb = open(path, "rb").read(128)
    assert sb[:8] == b"STRATA01"
    ver, flags = struct.unpack_from("<II", sb, 8)
    f8 = struct.unpack_from("<8Q", sb, 16)
    tix_off, tix_n = struct.unpack_from("<QQ", sb, 80)
    nl, ne, al = struct.unpack_from("<III", sb, 96)
    crc = struct.unpack_from("<I", sb, 108)[0]
    assert crc == zlib.crc32(sb[:108]) & 0xFFFFFFFF
    keys = ["meta_off", "meta_size", "index_off", "index_count", "trunk_off", "trunk_size", "expert_off",
            "expert_size"]
    return dict(zip(keys, f8), version=ver, flags=flags, tix_off=tix_off, tix_n=tix_n, n_layers=nl, n_experts=ne,
                align=al)


def _expect(src, cfg):
    """Trunk tensors and bundles of a stacked source, by name."""
    t = {n: d for n, _, _, d in src["tensors"]}
    trunk = {n: d for n, d in t.items() if "_exps." not in n}
    bundles = {}
    for l in range(cfg.n_layer):
        parts = [t[f"blk.{l}.ffn_{k}_exps.weight"] for k in ("gate", "up", "down")]
        for e in range(cfg.n_expert):
            bundles[(l, e)] = b"".join(p[e * (len(p) // cfg.n_expert):(e + 1) * (len(p) // cfg.n_expert)]
                                       for p in parts)
    return trunk, bundles


@pytest.mark.parametrize("alignment", [32, 64])
def test_pack_stacked_gguf_verbatim(model, tmp_path, alignment):
    from strataflow_b200.strata import StrataFile, pack
    cfg, om = model
    g, s = tmp_path / "m.gguf", tmp_path / "m.strata"
    src = write_gguf(g, om, cfg, alignment=alignment)
    pack(g, s)
    sb = _superblock(s)
    assert sb["version"] == 2 and sb["flags"] == 1 | 2 | 4 and sb["align"] == 4096
    assert sb["n_layers"] == cfg.n_layer and sb["n_experts"] == cfg.n_expert
    assert sb["index_count"] == cfg.n_layer * cfg.n_expert
    for k in ("trunk_off", "expert_off", "tix_off"):
        assert sb[k] % 4096 == 0, k
    raw = open(s, "rb").read()
    # the embedded metadata is the source's own prefix, byte for byte
    assert raw[sb["meta_off"]:sb["meta_off"] + sb["meta_size"]] == src["meta"]
    trunk, bundles = _expect(src, cfg)
    with StrataFile(s) as f:
        hp = f.hparams()
        assert (hp.n_embd, hp.n_layer, hp.n_expert, hp.n_ff, hp.n_vocab) == \
            (cfg.n_embd, cfg.n_layer, cfg.n_expert, cfg.n_ff, cfg.n_vocab)
        for name, data in trunk.items():
            assert f.read_trunk(name, len(data)).tobytes() == data, name
        for (l, e), b in bundles.items():
            assert f.read_bundle(l, e).tobytes() == b, (l, e)
    # every expert blob starts on a 4 KiB boundary; trunk tensors are back to back in source order
    ent = [struct.unpack_from("<IIQQQQQ", raw, sb["index_off"] + 48 * i) for i in range(sb["index_count"])]
    assert [(x[0], x[1]) for x in ent] == [(l, e) for l in range(cfg.n_layer) for e in range(cfg.n_expert)]
    assert all(x[2] % 4096 == 0 for x in ent)
    assert sum(len(d) for d in trunk.values()) == sb["trunk_size"]


def test_pack_is_deterministic(model, tmp_path):
    from strataflow_b200.strata import pack
    cfg, om = model
    g = tmp_path / "m.gguf"
    write_gguf(g, om, cfg)
    pack(g, tmp_path / "a.strata")
    pack(g, tmp_path / "b.strata")
    assert open(tmp_path / "a.strata", "rb").read() == open(tmp_path / "b.strata", "rb").read()


def test_pack_legacy_per_expert_gguf(model, tmp_path):
    """Per-expert tensors are regrouped: the same bundles as the stacked
    source, and metadata declaring stacked _exps tensors."""
    from strataflow_b200.strata import StrataFile, pack
    cfg, om = model
    stacked = write_gguf(tmp_path / "s.gguf", om, cfg)
    write_gguf(tmp_path / "l.gguf", om, cfg, legacy=True)
    pack(tmp_path / "l.gguf", tmp_path / "l.strata")
    trunk, bundles = _expect(stacked, cfg)
    with StrataFile(tmp_path / "l.strata") as f:
        names = {t["name"]: t for t in f.tensors()}
        for l in range(cfg.n_layer):
            for k in ("gate", "up", "down"):
                t = names[f"blk.{l}.ffn_{k}_exps.weight"]
                assert t["ne"][2] == cfg.n_expert
        assert not any(".ffn_gate.0." in n for n in names)
        for name, data in trunk.items():
            assert f.read_trunk(name, len(data)).tobytes() == data, name
        for (l, e), b in bundles.items():
            assert f.read_bundle(l, e).tobytes() == b, (l, e)
    sb = _superblock(tmp_path / "l.strata")
    assert sb["n_experts"] == cfg.n_expert and sb["n_layers"] == cfg.n_layer


def test_pack_refusals(model, tmp_path):
    from strataflow_b200.strata import pack
    cfg, om = model
    # the metadata declares experts but none is recognised by name
    write_gguf(tmp_path / "h.gguf", om, cfg, hide_experts=True)
    with pytest.raises(L.SfkError) as ei:
        pack(tmp_path / "h.gguf", tmp_path / "h.strata")
    assert ei.value.status == L.SFK_ERR_INVALID_ARGUMENT and b"no expert tensor" in L.load().sfk_last_error()
    assert not (tmp_path / "h.strata").exists()      # no partial output is left behind
    # stacked and per-expert tensors mixed
    write_gguf(tmp_path / "x.gguf", om, cfg, mix=True)
    with pytest.raises(L.SfkError) as ei:
        pack(tmp_path / "x.gguf", tmp_path / "x.strata")
    assert b"mixed" in L.load().sfk_last_error()
    # not a GGUF / truncated / missing
    (tmp_path / "bad.gguf").write_bytes(b"NOPE" + bytes(64))
    with pytest.raises(L.SfkError):
        pack(tmp_path / "bad.gguf", tmp_path / "bad.strata")
    src = open(tmp_path / "h.gguf", "rb").read()
    write_gguf(tmp_path / "ok.gguf", om, cfg)
    full = open(tmp_path / "ok.gguf", "rb").read()
    (tmp_path / "cut.gguf").write_bytes(full[:len(full) // 2])
    with pytest.raises(L.SfkError) as ei:
        pack(tmp_path / "cut.gguf", tmp_path / "cut.strata")
    assert b"outside the file" in L.load().sfk_last_error()
    with pytest.raises(L.SfkError):
        pack(tmp_path / "missing.gguf", tmp_path / "m.strata")
    assert len(src) > 0


def test_pack_command_line(model, tmp_path, capsys):
    from strataflow_b200 import strata_pack
    cfg, om = model
    write_gguf(tmp_path / "m.gguf", om, cfg)
    assert strata_pack.main([str(tmp_path / "m.gguf"), str(tmp_path / "m.strata")]) == 0
    assert "wrote" in capsys.readouterr().out
    assert strata_pack.main([str(tmp_path / "none.gguf"), str(tmp_path / "n.strata")]) == 1


@pytest.mark.gpu
@pytest.mark.parametrize("legacy,expert_slots", [(False, 0), (True, 5)])
def test_packed_gguf_decodes_like_the_oracle(cuda, model, tmp_path, legacy, expert_slots):
    """GGUF -> strata-pack -> Engine::load of the .strata (fully resident, and
    with a bounded expert tier): the HBM tier holds the oracle model's bytes
    and the greedy decode is the oracle's."""
    from strataflow_b200 import engine as E
    from strataflow_b200.strata import pack
    cfg, om = model
    write_gguf(tmp_path / "m.gguf", om, cfg, legacy=legacy)
    pack(tmp_path / "m.gguf", tmp_path / "m.strata")
    eng = E.Engine.load_strata(str(tmp_path / "m.strata"), kv_type=L.KV_F32, expert_slots=expert_slots)
    for tid, l in om.tensors():
        assert np.array_equal(eng.get(tid, l), om.tensor(tid, l)[0]), (tid, l)
    prompt = [5, 77, 1234, 4000, 9]
    toks, logits = eng.generate(prompt, 6, host_loop=True)
    o_toks, o_logits = O.greedy(om, prompt, 6, want_logits=True)
    assert toks == o_toks
    for a, b in zip(logits, o_logits):
        assert float(np.linalg.norm(a - b) / np.linalg.norm(b)) < 1e-3 and float(np.abs(a - b).max()) < 1e-2
    eng.close()
