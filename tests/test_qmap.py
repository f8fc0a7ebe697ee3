"""QMAP v1 blob consumption on the host (no GPU).

The C walker (q4gpu_qmap_read_packet / q4gpu_qmap_vector / q4gpu_qmap_bind)
is pinned against real packets the reference exported
(tests/golden/qmap_ref.npz, built by make_qmap_golden.py): their headers,
descriptor tables and parameter payloads (gammas, LUTs) must decode to the
reference's own stage vectors.  The writer's segment plan must equal the
deployed 61-segment plan, and a written image must bind back to the tensors
it was written from."""
from pathlib import Path

import numpy as np
import pytest

from llm_accelerator_b200 import _native, qmap, tables

GOLDEN = np.load(Path(__file__).parent / "golden" / "qmap_ref.npz")


def _packet(name):
    b = GOLDEN[f"pkt_{name}"]
    base = int(np.frombuffer(b[0x28:0x30].tobytes(), "<u8")[0])
    return b, base


def _param(name, nth):
    b, base = _packet(name)
    _, descs = qmap.read_packet(b, base, base)
    x = [d for d in descs if d["role"] == qmap.R_PARAM][nth]
    t = _native.QmapTensor()
    t.data_offset = x["base_addr"] - base
    t.elem_stride = x["strides_bytes"][0]
    t.rows = x["dims"][0]
    t.data_bytes = t.elem_stride * t.rows
    t.elem_kind = {qmap.DT_I16_Q8_7: _native.QMAP_S16, qmap.DT_U16_Q0_16: _native.QMAP_U16,
                   qmap.DT_U32_Q0_20: _native.QMAP_U32}[x["dtype"]]
    return qmap.vector(b, t)


@pytest.mark.parametrize("name", ["input_rmsnorm", "attn_frontend", "attn_score_value", "o_proj", "post_attn_norm",
                                  "mlp_gate_up", "mlp_silu_mul", "mlp_down", "mlp_residual_add", "qkv",
                                  "final_tail"])
def test_real_packet_headers(name):
    b, base = _packet(name)
    h, descs = qmap.read_packet(b, base, base)
    assert h["magic"] == qmap.MAGIC and h["version"] == 1
    assert h["header_bytes"] == 256 and h["descriptor_bytes"] == 128
    assert h["image_base_addr"] == base and h["descriptor_table_addr"] == base + 0x100
    assert h["payload_base_addr"] == base + 0x100 + 128 * h["descriptor_capacity"]
    assert len(descs) == h["descriptor_count"] <= h["descriptor_capacity"]
    assert descs[0]["role"] == qmap.R_META
    for d in descs:
        if d["role"] == qmap.R_WEIGHT:  # packed low-even Q4 with a scale in the same packet
            assert d["dtype"] == qmap.DT_PACKED_Q4 and d["flags"] & qmap.F_PACKED_LOW_EVEN
            assert d["strides_bytes"][0] == d["dims"][1] // 2
            s = [x for x in descs if x["tensor_id"] == d["scale_tensor_id"]]
            assert len(s) == 1 and s[0]["role"] == qmap.R_SCALE and s[0]["dims"] == [d["dims"][0], d["dims"][1] // 64,
                                                                                      0, 0]


def test_real_packet_slot_tables():
    roles = {n: [d["role"] for d in qmap.read_packet(*_packet(n), _packet(n)[1])[1]]
             for n in ("attn_frontend", "attn_score_value", "o_proj", "mlp_gate_up", "mlp_down", "final_tail")}
    R = qmap
    assert roles["attn_frontend"] == [R.R_META, R.R_ACT, R.R_ACT, R.R_ACT, R.R_PARAM, R.R_PARAM, R.R_ROPE, R.R_ROPE,
                                      R.R_KV, R.R_OUTPUT]
    assert roles["attn_score_value"] == [R.R_META, R.R_ACT, R.R_KV, R.R_PARAM, R.R_OUTPUT]
    assert roles["o_proj"][:5] == [R.R_META, R.R_ACT, R.R_WEIGHT, R.R_SCALE, R.R_OUTPUT]
    assert roles["mlp_gate_up"][:8] == [R.R_META, R.R_ACT, R.R_WEIGHT, R.R_SCALE, R.R_WEIGHT, R.R_SCALE, R.R_OUTPUT,
                                        R.R_OUTPUT]
    assert roles["final_tail"] == [R.R_META, R.R_ACT, R.R_WEIGHT, R.R_SCALE, R.R_OUTPUT, R.R_EXPECTED, R.R_ACT,
                                   R.R_PARAM]
    _, sv = qmap.read_packet(*_packet("attn_score_value"), _packet("attn_score_value")[1])
    assert sv[0]["aux"][0] == qmap.SCORE_SCALE_Q0_31


def test_real_packet_parameters_match_stage_vectors():
    assert np.array_equal(_param("input_rmsnorm", 0), GOLDEN["ref_input_gamma"])
    assert np.array_equal(_param("post_attn_norm", 0), GOLDEN["ref_post_gamma"])
    assert np.array_equal(_param("attn_frontend", 0), GOLDEN["ref_q_gamma"])
    assert np.array_equal(_param("attn_frontend", 1), GOLDEN["ref_k_gamma"])
    assert np.array_equal(_param("attn_score_value", 0), GOLDEN["ref_exp_lut"])
    assert np.array_equal(_param("mlp_silu_mul", 0), GOLDEN["ref_sigmoid_lut"])
    assert np.array_equal(_param("final_tail", 0), GOLDEN["ref_final_gamma"])


def test_real_packet_tables_match_ours():
    """The LUTs and the RoPE row in the reference's packets equal this build's
    table generators (the front-end packet's position is its metadata aux3)."""
    e, s = tables.luts()
    assert np.array_equal(e, GOLDEN["ref_exp_lut"]) and np.array_equal(s, GOLDEN["ref_sigmoid_lut"])
    b, base = _packet("attn_frontend")
    _, descs = qmap.read_packet(b, base, base)
    pos = descs[0]["aux"][3]
    cos, sin = tables.rope_tables(256)
    rope = [d for d in descs if d["role"] == qmap.R_ROPE]
    for plane, ref in zip(rope, (cos, sin)):
        v = np.frombuffer(b[plane["base_addr"] - base:plane["base_addr"] - base + 512].tobytes(), "<i4")
        assert np.array_equal(v, ref[pos])


def test_segment_plan_is_the_deployed_plan():
    plan = qmap.segment_plan(28, 151936)
    assert [s.address for s in plan] == GOLDEN["seg_address"].tolist()
    assert [s.nbytes for s in plan] == GOLDEN["seg_nbytes"].tolist()
    ops = {0: "file", 1: "zero"}
    ref = [(int(i), str(n), ops[int(o)], int(a), int(b)) for i, n, o, a, b in
           zip(GOLDEN["ent_segment"], GOLDEN["ent_name"], GOLDEN["ent_op"], GOLDEN["ent_address"],
               GOLDEN["ent_nbytes"])]
    ours = [(s.index,) + e for s in plan for e in s.entries]
    assert ours == ref
    assert [qmap.layer_bases(i)[0] for i in (0, 1, 27)] == [0x405000000, 0x405840000, 0x405000000 + 27 * 0x840000]
    assert qmap.layer_bases(0)[1:] == (0x4179A0000, 0x417920000, 0x417930000, 0x417940000, 0x417950000,
                                       0x417960000, 0x417970000, 0x417980000, 0x417990000)


def _random_tensors(n_layers=2, vocab=4096, seed=0):
    rng = np.random.default_rng(seed)
    t = qmap.ModelTensors(n_layers=n_layers)
    shapes = {_native.T_Q: (2048, 1024), _native.T_K: (1024, 1024), _native.T_V: (1024, 1024),
              _native.T_O: (1024, 2048), _native.T_GATE: (3072, 1024), _native.T_UP: (3072, 1024),
              _native.T_DOWN: (1024, 3072)}
    for layer in range(n_layers):
        for which, (r, c) in shapes.items():
            t.weights[(layer, which)] = (rng.integers(0, 256, (r, c // 2), dtype=np.uint8),
                                         rng.integers(0, 65536, (r, c // 64)).astype(np.uint16))
        for which, n in ((_native.T_INPUT_GAMMA, 1024), (_native.T_POST_GAMMA, 1024), (_native.T_Q_GAMMA, 128),
                         (_native.T_K_GAMMA, 128)):
            t.gammas[(layer, which)] = rng.integers(-32768, 32768, n).astype(np.int32)
    t.embed = (rng.integers(0, 256, (vocab, 512), dtype=np.uint8), rng.integers(0, 65536, (vocab, 16)).astype(np.uint16))
    t.final_gamma = rng.integers(-32768, 32768, 1024).astype(np.int32)
    t.rope_cos, t.rope_sin = tables.rope_tables(256)
    t.exp_lut, t.sig_lut = tables.luts()
    return t


@pytest.fixture(scope="module")
def written(tmp_path_factory):
    t = _random_tensors()
    segs = qmap.build_segments(t)
    man = qmap.write_bundle(segs, tmp_path_factory.mktemp("qmap"))
    arena, base = qmap.load_bundle(man)
    return t, segs, arena, base


def test_written_plan_and_packets(written):
    t, segs, arena, base = written
    assert [(s.address, s.nbytes, s.entries) for s in segs] == \
        [(s.address, s.nbytes, s.entries) for s in qmap.segment_plan(t.n_layers, t.vocab)]
    for layer in range(t.n_layers):
        for addr in qmap.layer_bases(layer):
            h, _ = qmap.read_packet(arena, base, addr)
            assert h["image_base_addr"] == addr


def test_bind_round_trip(written):
    t, _, arena, base = written
    bound = qmap.bind(arena, qmap.Layout(t.n_layers))
    assert len(bound) == 11 * t.n_layers + 6
    seen = set()
    for b in bound:
        seen.add((b.layer, b.which))
        if b.elem_kind == _native.QMAP_PACKED_Q4:
            w, s = t.embed if b.which == _native.T_EMBED else t.weights[(b.layer, b.which)]
            assert bytes(arena[b.data_offset:b.data_offset + b.data_bytes]) == w.tobytes()
            assert bytes(arena[b.scale_offset:b.scale_offset + b.scale_bytes]) == s.astype("<u2").tobytes()
            continue
        v = qmap.vector(arena, b)
        want = {_native.T_FINAL_GAMMA: t.final_gamma, _native.T_EXP_LUT: t.exp_lut, _native.T_SIGMOID_LUT: t.sig_lut,
                _native.T_ROPE_COS: t.rope_cos, _native.T_ROPE_SIN: t.rope_sin}.get(b.which)
        if want is None:
            want = t.gammas[(b.layer, b.which)]
        assert np.array_equal(v, np.asarray(want).reshape(-1))
    assert len(seen) == len(bound)


def _corrupt(arena, addr, offset, value, fmt="<I"):
    import struct
    a = arena.copy()
    struct.pack_into(fmt, a, addr - qmap.APERTURE_BASE + offset, value)
    return a


@pytest.mark.parametrize("what", ["magic", "matrix_id", "lut", "score_scale", "gamma_word"])
def test_bind_rejects_bad_images(written, what):
    t, _, arena, _ = written
    lay = qmap.Layout(t.n_layers)
    b1 = qmap.layer_bases(1)
    if what == "magic":
        bad = _corrupt(arena, b1[4], 0, 0x12345678)  # layer 1 o_proj packet
    elif what == "matrix_id":  # o_proj weight descriptor (slot 2) aux0 -> gate
        bad = _corrupt(arena, b1[4], 0x100 + 2 * 128 + 0x60, qmap.M_GATE)
    elif what == "lut":  # layer 1's exp LUT differs from layer 0's
        _, descs = qmap.read_packet(arena, qmap.APERTURE_BASE, b1[3])
        lut = [d for d in descs if d["role"] == qmap.R_PARAM][0]
        bad = _corrupt(arena, lut["base_addr"], 4, 12345)
    elif what == "score_scale":
        bad = _corrupt(arena, b1[3], 0x100 + 0x60, 189812530)
    else:  # a gamma word that is not a sign-extended 16-bit value
        _, descs = qmap.read_packet(arena, qmap.APERTURE_BASE, b1[1])
        g = [d for d in descs if d["role"] == qmap.R_PARAM][0]
        bad = _corrupt(arena, g["base_addr"], 0, 0x00012345)
        bound = qmap.bind(bad, lay)
        x = [b for b in bound if b.layer == 1 and b.which == _native.T_INPUT_GAMMA][0]
        with pytest.raises(_native.Q4GpuError):
            qmap.vector(bad, x)
        return
    with pytest.raises(_native.Q4GpuError):
        qmap.bind(bad, lay)


def test_load_bundle_checks(written, tmp_path):
    import json
    t, segs, _, _ = written
    man = qmap.write_bundle(segs, tmp_path)
    m = json.loads(man.read_text())
    m["segments"][1]["sha256"] = "0" * 64
    man.write_text(json.dumps(m))
    with pytest.raises(ValueError):
        qmap.load_bundle(man)
    m["segments"][1]["sha256"] = None
    m["segments"][2]["address"] = m["segments"][1]["address"] + 16  # overlap
    man.write_text(json.dumps(m))
    with pytest.raises(ValueError):
        qmap.load_bundle(man)
