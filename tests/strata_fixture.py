"""Write small .strata files for the loader tests (test infrastructure).

The layout is the reference's packed format (src/tws/strata_format.h:1-177,
packer tools/strata-pack):

    [128-byte superblock]
    [embedded GGUF metadata: header + key/values + tensor infos]
    [expert index: one 48-byte ExpertIndexEntry per (layer, expert)]
    [trunk block, 4 KiB-aligned: every non-expert tensor, GGUF order, no padding]
    [expert region, 4 KiB-aligned: one 4 KiB-aligned blob gate|up|down per (layer, expert)]
    [v2+: trunk index, 80-byte TrunkIndexEntry per trunk tensor]

Superblock trailing fields per version (strata_format.h:52-66): v1 n_layers@80;
v2 trunk_index_offset@80, trunk_index_count@88, n_layers@96; v3 adds
compress_index_offset@96, compress_index_count@104, n_layers@112.  The header
CRC32 (IEEE, zlib's) covers every byte before it.

Tensor bytes come from the CPU oracle's model (GGUF block layout), so a test
can load the same weights through the .strata path and through
sfk_weights_put and compare decodes.
"""
from __future__ import annotations

import struct
import zlib

import numpy as np

ALIGN = 4096
NAMES = {0: "token_embd.weight", 1: "output_norm.weight", 2: "output.weight", 3: "attn_norm.weight",
         4: "attn_q.weight", 5: "attn_k.weight", 6: "attn_v.weight", 7: "attn_output.weight", 8: "ffn_norm.weight",
         9: "ffn_gate_inp.weight", 10: "ffn_gate_exps.weight", 11: "ffn_up_exps.weight", 12: "ffn_down_exps.weight"}
LAYER_ORDER = (3, 4, 5, 6, 7, 8, 9, 10, 12, 11)   # llama.cpp's per-block order (gate, down, up)
EXPERT_TIDS = (10, 11, 12)


def _gstr(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _kv(key: str, vtype: int, payload: bytes) -> bytes:
    return _gstr(key) + struct.pack("<I", vtype) + payload


def gguf_meta(model, cfg) -> tuple[bytes, list]:
    """GGUF v3 header + key/values + tensor infos; returns (blob, tensor list
    [(name, tid, layer, type, ne, bytes)] in GGUF order)."""
    tensors = [("token_embd.weight", 0, 0)]
    for l in range(cfg.n_layer):
        tensors += [(f"blk.{l}.{NAMES[t]}", t, l) for t in LAYER_ORDER]
    tensors += [("output_norm.weight", 1, 0), ("output.weight", 2, 0)]
    out = []
    for name, tid, layer in tensors:
        data, qtype, ne = model.tensor(tid, layer)
        out.append((name, tid, layer, qtype, ne, np.array(data, copy=True)))
    kvs = [
        _kv("general.architecture", 8, _gstr("llama")),
        _kv("llama.block_count", 4, struct.pack("<I", cfg.n_layer)),
        _kv("llama.context_length", 4, struct.pack("<I", cfg.n_ctx)),
        _kv("llama.embedding_length", 4, struct.pack("<I", cfg.n_embd)),
        _kv("llama.feed_forward_length", 4, struct.pack("<I", cfg.n_ff)),
        _kv("llama.attention.head_count", 4, struct.pack("<I", cfg.n_head)),
        _kv("llama.attention.head_count_kv", 5, struct.pack("<i", cfg.n_head_kv)),   # an i32 key on purpose
        _kv("llama.expert_count", 4, struct.pack("<I", cfg.n_expert)),
        _kv("llama.expert_used_count", 4, struct.pack("<I", cfg.n_expert_used)),
        _kv("llama.attention.layer_norm_rms_epsilon", 6, struct.pack("<f", cfg.rms_eps)),
        _kv("llama.rope.freq_base", 6, struct.pack("<f", cfg.freq_base)),
        # an array of strings and one of u32, as a tokenizer block carries
        _kv("tokenizer.ggml.tokens", 9, struct.pack("<IQ", 8, 3) + _gstr("<s>") + _gstr("</s>") + _gstr("a")),
        _kv("tokenizer.ggml.token_type", 9, struct.pack("<IQ", 4, 3) + struct.pack("<3I", 1, 1, 1)),
    ]
    blob = b"GGUF" + struct.pack("<IQQ", 3, len(out), len(kvs)) + b"".join(kvs)
    off = 0
    for name, _, _, qtype, ne, data in out:
        dims = list(ne)
        while len(dims) > 1 and dims[-1] == 1:
            dims.pop()
        blob += _gstr(name) + struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}Q", *dims)
        blob += struct.pack("<IQ", qtype, off)
        off += (data.nbytes + 31) // 32 * 32
    return blob, out


def _pad(buf: bytearray, align: int = ALIGN) -> None:
    buf.extend(b"\0" * ((-len(buf)) % align))


def write_strata(path, model, cfg, version: int = 2, compressed_flag: bool = False,
                 corrupt_trunk_index: bool = False) -> dict:
    """Pack `model` (an oracle Model of shape `cfg`) into a .strata file.
    Returns the expected contents: {"trunk": {name: bytes}, "bundles": {(l, e): bytes}}."""
    meta, tensors = gguf_meta(model, cfg)
    E = cfg.n_expert
    bundles = {}
    stacks = {(tid, l): data for _, tid, l, _, _, data in tensors if tid in EXPERT_TIDS}
    for l in range(cfg.n_layer):
        for e in range(E):
            parts = []
            for tid in EXPERT_TIDS:
                d = stacks[(tid, l)]
                per = d.nbytes // E
                parts.append(d[e * per:(e + 1) * per].tobytes())
            bundles[(l, e)] = parts
    trunk = [(name, data) for name, tid, _, _, _, data in tensors if tid not in EXPERT_TIDS]

    f = bytearray(b"\0" * 128)
    meta_off = len(f)
    f += meta
    index_off = len(f)
    n_index = cfg.n_layer * E
    f += b"\0" * (48 * n_index)
    _pad(f)
    trunk_off = len(f)
    rel = {}
    for name, data in trunk:
        rel[name] = len(f) - trunk_off
        f += data.tobytes()
    trunk_size = len(f) - trunk_off
    _pad(f)
    expert_off = len(f)
    entries = []
    for (l, e), (g, u, d) in sorted(bundles.items()):
        _pad(f)
        off = len(f)
        f += g + u + d
        entries.append(struct.pack("<IIQQQQQ", l, e, off, len(g) + len(u) + len(d), 0, len(g), len(g) + len(u)))
    expert_size = len(f) - expert_off
    f[index_off:index_off + 48 * n_index] = b"".join(entries)
    tix_off, tix_n = 0, 0
    if version >= 2:
        _pad(f, 8)
        tix_off, tix_n = len(f), len(trunk)
        for name, data in trunk:
            r = rel[name] + (16 if corrupt_trunk_index and name == "output.weight" else 0)
            f += name.encode().ljust(64, b"\0") + struct.pack("<QQ", r, data.nbytes)
    flags = 1 | 2 | (4 if tix_n else 0) | (8 if compressed_flag else 0)
    sb = b"STRATA01" + struct.pack("<II", version, flags)
    sb += struct.pack("<8Q", meta_off, len(meta), index_off, n_index, trunk_off, trunk_size, expert_off, expert_size)
    if version >= 2:
        sb += struct.pack("<QQ", tix_off, tix_n)
    if version >= 3:
        sb += struct.pack("<QQ", 0, 0)
    sb += struct.pack("<III", cfg.n_layer, E, ALIGN)
    sb += struct.pack("<I", zlib.crc32(sb) & 0xFFFFFFFF)
    assert len(sb) <= 128
    f[0:len(sb)] = sb
    with open(path, "wb") as fh:
        fh.write(bytes(f))
    return {"trunk": {n: d.tobytes() for n, d in trunk},
            "bundles": {k: b"".join(v) for k, v in bundles.items()},
            "tensors": [(n, t, l, q, ne) for n, t, l, q, ne, _ in tensors]}


def write_gguf(path, model, cfg, legacy: bool = False, alignment: int = 32, hide_experts: bool = False,
               mix: bool = False) -> dict:
    """A whole GGUF file (metadata + aligned data section) of `model`, the
    input of the product packer.  legacy: the experts as per-expert 2-D
    tensors blk.L.ffn_{gate,up,down}.E.weight (the old Mixtral naming);
    hide_experts: expert tensors renamed so nothing recognises them; mix:
    layer 0 stacked, the others per-expert.  Returns the source layout:
    {"data_offset", "meta", "tensors": [(name, type, ne, bytes)]}."""
    _, tensors = gguf_meta(model, cfg)
    E = cfg.n_expert
    kind = {10: "ffn_gate", 11: "ffn_up", 12: "ffn_down"}
    out = []
    for name, tid, layer, qtype, ne, data in tensors:
        per_expert = tid in EXPERT_TIDS and (legacy or (mix and layer > 0))
        if per_expert:
            per = data.nbytes // E
            for e in range(E):
                out.append((f"blk.{layer}.{kind[tid]}.{e}.weight", qtype, [ne[0], ne[1]],
                            data.view(np.uint8)[e * per:(e + 1) * per].copy()))
        else:
            nm = name.replace("_exps.", "_xps.") if hide_experts and tid in EXPERT_TIDS else name
            out.append((nm, qtype, list(ne), data))
    kvs = [
        _kv("general.architecture", 8, _gstr("llama")),
        _kv("general.alignment", 4, struct.pack("<I", alignment)),
        _kv("llama.block_count", 4, struct.pack("<I", cfg.n_layer)),
        _kv("llama.context_length", 4, struct.pack("<I", cfg.n_ctx)),
        _kv("llama.embedding_length", 4, struct.pack("<I", cfg.n_embd)),
        _kv("llama.feed_forward_length", 4, struct.pack("<I", cfg.n_ff)),
        _kv("llama.attention.head_count", 4, struct.pack("<I", cfg.n_head)),
        _kv("llama.attention.head_count_kv", 4, struct.pack("<I", cfg.n_head_kv)),
        _kv("llama.expert_count", 4, struct.pack("<I", cfg.n_expert)),
        _kv("llama.expert_used_count", 4, struct.pack("<I", cfg.n_expert_used)),
        _kv("llama.attention.layer_norm_rms_epsilon", 6, struct.pack("<f", cfg.rms_eps)),
        _kv("llama.rope.freq_base", 6, struct.pack("<f", cfg.freq_base)),
        _kv("tokenizer.ggml.tokens", 9, struct.pack("<IQ", 8, 3) + _gstr("<s>") + _gstr("</s>") + _gstr("a")),
    ]
    meta = b"GGUF" + struct.pack("<IQQ", 3, len(out), len(kvs)) + b"".join(kvs)
    off = 0
    offs = []
    for name, qtype, ne, data in out:
        dims = list(ne)
        while len(dims) > 1 and dims[-1] == 1:
            dims.pop()
        meta += _gstr(name) + struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}Q", *dims)
        meta += struct.pack("<IQ", qtype, off)
        offs.append(off)
        off += (data.nbytes + alignment - 1) // alignment * alignment
    data_offset = (len(meta) + alignment - 1) // alignment * alignment
    f = bytearray(meta) + b"\0" * (data_offset - len(meta))
    for (name, qtype, ne, data), o in zip(out, offs):
        f += b"\0" * (data_offset + o - len(f))
        f += data.tobytes()
    with open(path, "wb") as fh:
        fh.write(bytes(f))
    return {"data_offset": data_offset, "meta": bytes(f[:data_offset]),
            "tensors": [(n, q, ne, d.tobytes()) for n, q, ne, d in out]}
