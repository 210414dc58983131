"""GGUF loader (srhpm_b200.gguf) and the tensor-parallel slicing it shares with the verify step.

The files are written by gguf-py's GGUFWriter (an independent implementation of the format). The parser must return
the same metadata, shapes, types and bytes. Slices of every rank must tile each matrix exactly:
- rows for the column-parallel QKV / gate / up / head;
- block-aligned column ranges for the row-parallel O / down.
CPU only: the device upload path is covered by tests/test_verify_step_gpu.py."""
import numpy as np
import pytest

gguf_py = pytest.importorskip("gguf")

import srhpm_b200 as S
from srhpm_b200 import gguf as G
from srhpm_b200 import shard
from srhpm_b200 import verify_step as V


def small_cfg():
    return V.DecoderConfig(n_layer=2, d=512, n_ff=1024, H=4, Hkv=2, hd=128, n_vocab=300, base=1e6, eps=1e-5,
                           window=0, full_every=1)


def write_decoder_gguf(path, cfg, w, arch="qwen2", qkv_split_types=False, extra_u32=None):
    """A llama.cpp-style dense decoder file from host_weights `w` (fused QKV rows split back into attn_q / k / v);
    extra_u32: more uint32 metadata {key: value}."""
    wr = gguf_py.GGUFWriter(str(path), arch)
    for key, val in (extra_u32 or {}).items():
        wr.add_uint32(key, val)
    wr.add_block_count(cfg.n_layer)
    wr.add_embedding_length(cfg.d)
    wr.add_feed_forward_length(cfg.n_ff)
    wr.add_head_count(cfg.H)
    wr.add_head_count_kv(cfg.Hkv)
    wr.add_key_length(cfg.hd)
    wr.add_value_length(cfg.hd)
    wr.add_rope_freq_base(cfg.base)
    wr.add_layer_norm_rms_eps(cfg.eps)
    wr.add_string("general.name", "synthetic")

    def q(name, blocks, qtype, rows, K):
        # gguf-py takes quantized tensors as their byte shape [rows, row bytes] and derives ne = [K, rows]
        wr.add_tensor(name, np.ascontiguousarray(blocks).reshape(rows, -1),
                      raw_dtype=gguf_py.GGMLQuantizationType(qtype))

    hd, H, Hkv = cfg.hd, cfg.H, cfg.Hkv
    wr.add_tensor("token_embd.weight", w["emb"])
    for l in range(cfg.n_layer):
        qkv = np.asarray(w["qkv"][l]).reshape((H + 2 * Hkv) * hd, -1)
        q(f"blk.{l}.attn_q.weight", qkv[:H * hd], cfg.types["qkv"], H * hd, cfg.d)
        q(f"blk.{l}.attn_k.weight", qkv[H * hd:(H + Hkv) * hd], cfg.types["qkv"], Hkv * hd, cfg.d)
        if qkv_split_types:  # V in another type: the loader must keep Q, K, V as separate GEMMs
            vf = np.random.default_rng(l).standard_normal((Hkv * hd, cfg.d)).astype(np.float32) * 0.02
            q(f"blk.{l}.attn_v.weight", S.quantize_chunk(vf, S.Q6_K), S.Q6_K, Hkv * hd, cfg.d)
        else:
            q(f"blk.{l}.attn_v.weight", qkv[(H + Hkv) * hd:], cfg.types["qkv"], Hkv * hd, cfg.d)
        q(f"blk.{l}.attn_output.weight", w["o"][l], cfg.types["o"], cfg.d, H * hd)
        q(f"blk.{l}.ffn_gate.weight", w["gate"][l], cfg.types["gate"], cfg.n_ff, cfg.d)
        q(f"blk.{l}.ffn_up.weight", w["up"][l], cfg.types["up"], cfg.n_ff, cfg.d)
        q(f"blk.{l}.ffn_down.weight", w["down"][l], cfg.types["down"], cfg.d, cfg.n_ff)
        wr.add_tensor(f"blk.{l}.attn_norm.weight", w["attn_norm"][l])
        wr.add_tensor(f"blk.{l}.ffn_norm.weight", w["ffn_norm"][l])
    wr.add_tensor("output_norm.weight", w["out_norm"])
    q("output.weight", w["head"], cfg.types["head"], cfg.n_vocab, cfg.d)
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    cfg = small_cfg()
    w = V.host_weights(cfg, seed=7)
    path = tmp_path_factory.mktemp("gguf") / "tiny.gguf"
    write_decoder_gguf(path, cfg, w)
    return cfg, w, path


def test_parse_metadata_and_config(model):
    cfg, w, path = model
    gf = G.GGUFFile(path)
    assert gf.version == 3
    assert gf.kv["general.architecture"] == "qwen2"
    assert gf.kv["general.name"] == "synthetic"
    assert gf.kv["qwen2.block_count"] == cfg.n_layer
    c = G.decoder_config(gf)
    for k in ("n_layer", "d", "n_ff", "H", "Hkv", "hd", "n_vocab"):
        assert getattr(c, k) == getattr(cfg, k), k
    assert c.base == pytest.approx(cfg.base) and c.eps == pytest.approx(cfg.eps)
    assert c.window == 0 and c.full_every == 1
    assert c.types == cfg.types
    gf.close()


def test_tensor_bytes_and_shapes(model):
    cfg, w, path = model
    gf = G.GGUFFile(path)
    t = gf.tensors["blk.1.ffn_down.weight"]
    assert t.ne == [cfg.n_ff, cfg.d] and t.type == cfg.types["down"]
    assert np.array_equal(gf.data("blk.1.ffn_down.weight"), np.asarray(w["down"][1]).reshape(cfg.d, -1))
    assert np.array_equal(gf.data("output.weight"), np.asarray(w["head"]).reshape(cfg.n_vocab, -1))
    assert np.array_equal(gf.data("token_embd.weight").view(np.float16).reshape(cfg.n_vocab, cfg.d), w["emb"])
    assert np.array_equal(gf.data("blk.0.attn_norm.weight").view(np.float32).reshape(-1), w["attn_norm"][0])
    qkv = np.asarray(w["qkv"][0]).reshape((cfg.H + 2 * cfg.Hkv) * cfg.hd, -1)
    assert np.array_equal(gf.data("blk.0.attn_k.weight"), qkv[cfg.H * cfg.hd:(cfg.H + cfg.Hkv) * cfg.hd])
    gf.close()


def test_not_gguf(tmp_path):
    p = tmp_path / "x.bin"
    p.write_bytes(b"NOPE" + bytes(60))
    with pytest.raises(ValueError):
        G.GGUFFile(p)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_tp_layout_tiles_the_model(world):
    H, Hkv, n_ff, n_vocab = 24, 4, 17408, 151936
    lays = [shard.tp_layout(H, Hkv, n_ff, n_vocab, world, r) for r in range(world)]
    # query heads, FFN rows and vocabulary rows partition their ranges
    for a, b in (("h0", "h1"), ("f0", "f1"), ("v0", "v1")):
        assert lays[0][a] == 0 and all(lays[i][b] == lays[i + 1][a] for i in range(world - 1))
    assert lays[-1]["h1"] == H and lays[-1]["f1"] == n_ff and lays[-1]["v1"] == n_vocab
    assert all(l["f0"] % 256 == 0 and l["f1"] % 256 == 0 for l in lays)
    G_ = H // Hkv
    for l in lays:  # every rank holds the KV heads of its query heads
        assert l["g0"] * G_ <= l["h0"] and l["h1"] <= l["g1"] * G_
    kv = sorted({(l["g0"], l["g1"]) for l in lays})
    assert kv[0][0] == 0 and kv[-1][1] == Hkv


def test_tp_layout_rejects_bad_splits():
    with pytest.raises(ValueError):
        shard.tp_layout(24, 4, 17408, 151936, 5, 0)
    with pytest.raises(ValueError):
        shard.tp_layout(24, 4, 17408, 151936, 3, 0)  # 4 KV heads on 3 ranks


def test_k_columns_tile_rows(model):
    cfg, w, path = model
    gf = G.GGUFFile(path)
    full = gf.data("blk.0.ffn_down.weight")
    t = gf.tensors["blk.0.ffn_down.weight"].type
    for world in (2, 4):
        parts = [G.k_columns(full, t, *shard.k_range(cfg.n_ff, world, r)) for r in range(world)]
        assert np.array_equal(np.concatenate(parts, axis=1), full)
    with pytest.raises(ValueError):
        G.k_columns(full, t, 100, 512)
    gf.close()


def test_split_types_detected(tmp_path):
    cfg = small_cfg()
    w = V.host_weights(cfg, seed=8)
    path = tmp_path / "split.gguf"
    write_decoder_gguf(path, cfg, w, qkv_split_types=True)
    gf = G.GGUFFile(path)
    assert gf.tensors["blk.0.attn_v.weight"].type == S.Q6_K
    assert gf.tensors["blk.0.attn_q.weight"].type == cfg.types["qkv"]
    gf.close()


def test_version_2_reads_like_3_and_others_are_refused(model, tmp_path):
    """GGUF v2 has v3's layout (64-bit counts and string lengths; v3 only added big-endian files): the same file with
    its version field set to 2 parses to the same metadata, tensor infos and bytes. Version 1 (32-bit counts) and
    unknown versions are refused, and so is a file cut inside its header."""
    import struct
    cfg, w, path = model
    raw = bytearray(open(path, "rb").read())
    a = G.GGUFFile(path)
    for ver, ok in ((2, True), (1, False), (4, False)):
        raw[4:8] = struct.pack("<I", ver)
        p = tmp_path / f"v{ver}.gguf"
        p.write_bytes(bytes(raw))
        if ok:
            b = G.GGUFFile(p)
            assert b.version == 2 and b.kv == a.kv and b.data_start == a.data_start
            assert {n: (t.ne, t.type, t.offset) for n, t in b.tensors.items()} == \
                   {n: (t.ne, t.type, t.offset) for n, t in a.tensors.items()}
            assert np.array_equal(b.data("output.weight"), a.data("output.weight"))
            b.close()
        else:
            with pytest.raises(ValueError):
                G.GGUFFile(p)
    raw[4:8] = struct.pack("<I", 3)
    cut = tmp_path / "cut.gguf"
    cut.write_bytes(bytes(raw[:200]))  # inside the key-value section
    with pytest.raises(ValueError):
        G.GGUFFile(cut)
    a.close()


def test_sliding_window_metadata(tmp_path):
    """`<arch>.attention.sliding_window` sets the window of the sliding layers; full attention then comes every 4th
    layer unless `full_every` says otherwise; explicit arguments override the file."""
    cfg = small_cfg()
    w = V.host_weights(cfg, seed=9)
    path = tmp_path / "swa.gguf"
    write_decoder_gguf(path, cfg, w, extra_u32={"qwen2.attention.sliding_window": 4096})
    gf = G.GGUFFile(path)
    assert gf.kv["qwen2.attention.sliding_window"] == 4096
    c = G.decoder_config(gf)
    assert c.window == 4096 and c.full_every == 4
    c2 = G.decoder_config(gf, window=0)
    assert c2.window == 0 and c2.full_every == 1
    c3 = G.decoder_config(gf, full_every=2)
    assert c3.window == 4096 and c3.full_every == 2
    gf.close()
