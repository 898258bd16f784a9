""".strata loader: the reader (host-only, runs on CPU) and the HBM load path
(GPU).  Files are packed by tests/strata_fixture.py in the reference's
on-disk layout (src/tws/strata_format.h) from the CPU oracle's weights; the
reference's own packer and reader tests (tests/test_strata_*.cpp) build their
fixtures the same way, at test time.
"""
import numpy as np
import pytest

from oracle import oracle as O
from strataflow_b200 import lib as L
from tests.strata_fixture import write_strata


def _cfg(**kw):
    d = dict(n_embd=256, n_head=8, n_head_kv=4, n_layer=2, n_ff=512, n_expert=8, n_expert_used=2, n_vocab=4096,
             n_ctx=80, rms_eps=1e-5, freq_base=10000.0)
    d.update(kw)
    return O.ModelConfig(**d)


@pytest.fixture(scope="module")
def packed(tmp_path_factory):
    """One file per superblock version, plus the oracle model behind them."""
    cfg = _cfg(type_ffn_gu=O.Q4_K, type_ffn_down=O.Q6_K, type_attn=O.Q8_0)
    om = O.Model(cfg, seed=21)
    d = tmp_path_factory.mktemp("strata")
    out = {}
    for v in (1, 2, 3):
        p = d / f"tiny_v{v}.strata"
        out[v] = (str(p), write_strata(p, om, cfg, version=v))
    return cfg, om, out


@pytest.mark.parametrize("version", [1, 2, 3])
def test_reader_hparams_and_tensor_table(packed, version):
    from strataflow_b200.strata import StrataFile
    cfg, _, files = packed
    path, want = files[version]
    with StrataFile(path) as f:
        hp = f.hparams()
        for k in ("n_embd", "n_head", "n_head_kv", "n_layer", "n_ff", "n_expert", "n_expert_used", "n_vocab",
                  "n_ctx", "type_embd", "type_attn", "type_ffn_gu", "type_ffn_down", "type_output"):
            assert getattr(hp, k) == getattr(cfg, k), k
        assert hp.rms_eps == np.float32(cfg.rms_eps) and hp.freq_base == np.float32(cfg.freq_base)
        table = f.tensors()
        assert [t["name"] for t in table] == [n for n, *_ in want["tensors"]]
        for t, (_, tid, _, qtype, ne) in zip(table, want["tensors"]):
            assert t["type"] == qtype and t["ne"][:3] == tuple(ne)
            assert t["expert"] == (tid in (10, 11, 12))


@pytest.mark.parametrize("version", [1, 2, 3])
def test_reader_trunk_and_bundles_are_verbatim(packed, version):
    from strataflow_b200.strata import StrataFile
    cfg, _, files = packed
    path, want = files[version]
    with StrataFile(path) as f:
        for name, data in want["trunk"].items():
            assert f.read_trunk(name, len(data)).tobytes() == data, name
        for (l, e), data in want["bundles"].items():
            assert f.read_bundle(l, e).tobytes() == data, (l, e)


def test_reader_rejects_damaged_files(packed, tmp_path):
    from strataflow_b200.strata import StrataFile
    cfg, om, files = packed
    good = open(files[2][0], "rb").read()

    def bad(blob, status, words):
        p = tmp_path / "bad.strata"
        p.write_bytes(blob)
        with pytest.raises(L.SfkError) as ei:
            StrataFile(str(p))
        assert ei.value.status == status
        assert any(w in str(ei.value) for w in words), str(ei.value)

    bad(b"GGUF" + good[4:], L.SFK_ERR_INVALID_ARGUMENT, ["magic"])
    flipped = bytearray(good)
    flipped[20] ^= 1                     # a field under the header CRC
    bad(bytes(flipped), 1, ["CRC"])
    bad(good[:100], 1, ["superblock"])
    bad(good[:len(good) // 2], 1, ["outside"])
    p = tmp_path / "comp.strata"
    write_strata(p, om, cfg, version=3, compressed_flag=True)
    bad(p.read_bytes(), L.SFK_ERR_UNSUPPORTED, ["compressed"])
    p = tmp_path / "tix.strata"
    write_strata(p, om, cfg, version=2, corrupt_trunk_index=True)
    bad(p.read_bytes(), 1, ["trunk index"])
    with pytest.raises(L.SfkError):
        StrataFile(str(tmp_path / "missing.strata"))


def test_reader_bundle_lookup_errors(packed):
    from strataflow_b200.strata import StrataFile
    cfg, _, files = packed
    with StrataFile(files[1][0]) as f:
        with pytest.raises(L.SfkError):
            f.read_bundle(cfg.n_layer, 0)      # no such layer
        with pytest.raises(L.SfkError):
            f.read_bundle(0, cfg.n_expert)     # no such expert
        with pytest.raises(L.SfkError):
            f.read_trunk("blk.0.ffn_gate_exps.weight", 16)   # an expert tensor is not in the trunk


@pytest.mark.gpu
@pytest.mark.parametrize("version", [1, 3])
def test_strata_load_decodes_like_the_same_weights_put_directly(cuda, packed, version):
    """Engine::load of a .strata file: the HBM tier holds the same bytes as
    when the tensors are uploaded one by one, and the greedy decode matches
    that engine bit for bit and the CPU oracle within the north-star bound."""
    from strataflow_b200 import engine as E
    cfg, om, files = packed
    path, _ = files[version]
    eng = E.Engine.load_strata(path, kv_type=L.KV_F32)
    ref_cfg = E.ModelConfig(**{k: getattr(eng.cfg, k) for k in E.ModelConfig.__dataclass_fields__})
    tensors = []
    for tid, l in om.tensors():
        data, qtype, ne = om.tensor(tid, l)
        tensors.append((tid, l, qtype, ne, data))
    ref = E.Engine.load(ref_cfg, tensors=tensors)
    for tid, l in om.tensors():
        assert np.array_equal(eng.get(tid, l), om.tensor(tid, l)[0]), (tid, l)
    prompt = [5, 77, 1234, 4000, 9]
    toks, logits = eng.generate(prompt, 6, host_loop=True)
    toks_r, logits_r = ref.generate(prompt, 6, host_loop=True)
    assert toks == toks_r
    for a, b in zip(logits, logits_r):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    o_toks, o_logits = O.greedy(om, prompt, 6, want_logits=True)
    assert toks == o_toks
    for a, b in zip(logits, o_logits):
        assert float(np.linalg.norm(a - b) / np.linalg.norm(b)) < 1e-3 and float(np.abs(a - b).max()) < 1e-2
    eng.close()
    ref.close()


@pytest.mark.gpu
@pytest.mark.parametrize("rank", [0, 1])
def test_strata_load_into_an_expert_parallel_engine(cuda, tmp_path, rank):
    """One rank of a two-rank engine loaded from a .strata file holds its own
    experts and, with the heads split (16 query / 4 kv heads of width 32: a
    rank's 8 query heads are 256 whole columns), its heads' rows of Q, K, V
    and its heads' columns of the output projection; the rest in full.  (The
    ranks are loaded one after the other on one GPU: loading needs no peer.)"""
    from strataflow_b200 import engine as E
    cfg = _cfg(n_embd=512, n_head=16, n_head_kv=4, n_layer=2, type_ffn_gu=O.Q4_K, type_ffn_down=O.Q8_0)
    om = O.Model(cfg, seed=13)
    path = tmp_path / "wide.strata"
    write_strata(path, om, cfg, version=2)
    eng = E.Engine.load_strata(str(path), kv_type=L.KV_F32, ep_size=2, ep_rank=rank)
    hd, hq, hkv, E_loc = 32, 8, 2, 4
    for l in range(cfg.n_layer):
        for tid, h0, hn in ((O.T_ATTN_Q, rank * hq, hq), (O.T_ATTN_K, rank * hkv, hkv), (O.T_ATTN_V, rank * hkv, hkv)):
            full, qtype, ne = om.tensor(tid, l)
            rows = full.reshape(ne[1], -1)
            assert np.array_equal(eng.get(tid, l), rows[h0 * hd:(h0 + hn) * hd].ravel()), (tid, l)
        full, qtype, ne = om.tensor(O.T_ATTN_OUT, l)                 # [d rows][Hq*hd columns]
        rb = O.row_bytes(qtype, hq * hd)
        want = full.reshape(ne[1], -1)[:, rank * rb:(rank + 1) * rb].ravel()
        assert np.array_equal(eng.get(O.T_ATTN_OUT, l), want), l
        for tid in (O.T_FFN_GATE_EXPS, O.T_FFN_UP_EXPS, O.T_FFN_DOWN_EXPS):
            full, _, _ = om.tensor(tid, l)
            experts = full.reshape(cfg.n_expert, -1)
            assert np.array_equal(eng.get(tid, l), experts[rank * E_loc:(rank + 1) * E_loc].ravel()), (tid, l)
        for tid in (O.T_ATTN_NORM, O.T_FFN_NORM, O.T_FFN_GATE_INP):
            assert np.array_equal(eng.get(tid, l), om.tensor(tid, l)[0]), (tid, l)
    for tid in (O.T_TOK_EMBD, O.T_OUTPUT_NORM, O.T_OUTPUT):
        assert np.array_equal(eng.get(tid, 0), om.tensor(tid, 0)[0]), tid
    eng.close()
