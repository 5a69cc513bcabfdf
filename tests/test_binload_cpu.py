"""The .bin weight-file reader (moe_bin_layer_info) and the tests' .bin writer,
against layer_ref.bin, which the reference's own exporter wrote
(tests/golden/make_golden.py bin; export.py:8-21, :188-206). Host only."""
import os

import numpy as np
import pytest

import moe_cuda as mc
from helpers import GOLDEN, synth, quant, write_bin, layer_records
from oracle.oracle import quantize_q8

REF_BIN = os.path.join(GOLDEN, "layer_ref.bin")


def ref_records():
    """The records of layer_ref.bin, rebuilt with the numpy quantisers."""
    recs = [("model.norm.weight", synth(60, 32, 1.0))]
    for layer, dt, bias, rname in ((1, 2, False, "mlp.gate.weight"), (3, 3, True, "mlp.router.gate.weight")):
        E, D, F = 3, 32, 16
        pre = f"model.layers.{layer}."
        recs.append((pre + rname, synth(61 + layer, E * D, 0.02).reshape(E, D)))
        if bias:
            recs.append((pre + "mlp.gate.bias", synth(62 + layer, E, 1.0)))
        q = "q8" if dt == 2 else "q4"
        for e in range(E):
            for j, (proj, rows, cols) in enumerate((("gate_proj", F, D), ("up_proj", F, D), ("down_proj", D, F))):
                s, qq = quant(dt)(synth(700 + 10 * layer + 3 * e + j, rows * cols, 0.02).reshape(rows, cols))
                base = f"{pre}mlp.experts.{e}.{proj}.weight"
                recs += [(base + ".scale", s), (base + "." + q, qq)]
    recs.append(("model.norm.weight", np.zeros(32, np.float32)))
    return recs


def test_writer_matches_reference_exporter(tmp_path):
    p = tmp_path / "w.bin"
    write_bin(str(p), ref_records())
    assert p.read_bytes() == open(REF_BIN, "rb").read()


def test_info_reference_file():
    assert mc.bin_layer_info(REF_BIN, 1) == (3, 32, 16, mc.Q8, 0)
    assert mc.bin_layer_info(REF_BIN, 3) == (3, 32, 16, mc.Q4, 1)


@pytest.mark.parametrize("layer", [0, 2, 4, -1])
def test_info_missing_layer(layer):
    with pytest.raises(mc.MoeError) as ei:
        mc.bin_layer_info(REF_BIN, layer)
    assert ei.value.code == mc.MOE_ERR_INVALID


def test_bad_magic_and_missing_file(tmp_path):
    p = tmp_path / "bad.bin"
    data = bytearray(open(REF_BIN, "rb").read())
    data[5] = 2                                          # version byte
    p.write_bytes(bytes(data))
    for path in (str(p), str(tmp_path / "absent.bin")):
        with pytest.raises(mc.MoeError) as ei:
            mc.bin_layer_info(path, 1)
        assert ei.value.code == mc.MOE_ERR_INVALID


def test_truncations_are_errors(tmp_path):
    """Every cut inside a record is reported, never read past (the reference
    exits on a short read, io.c:176-187). A cut exactly between records is a
    shorter valid file."""
    data = open(REF_BIN, "rb").read()
    p = tmp_path / "cut.bin"
    rng = np.random.default_rng(5)
    cuts = sorted(set([3, 9, 10, 12, 30] + list(rng.integers(11, len(data) - 1, 60))))
    for n in cuts:
        p.write_bytes(data[:n])
        try:
            info = mc.bin_layer_info(str(p), 3)
        except mc.MoeError as e:
            assert e.code == mc.MOE_ERR_INVALID
        else:
            # only possible when the cut fell after layer 3's last record
            assert info == (3, 32, 16, mc.Q4, 1) and n >= len(data) - 300


def test_count_field_not_authoritative(tmp_path):
    p = tmp_path / "c.bin"
    write_bin(str(p), ref_records(), count=1)           # io.c:212-233 reads to end of file
    assert mc.bin_layer_info(str(p), 3) == (3, 32, 16, mc.Q4, 1)


def test_unquantised_experts_unsupported(tmp_path):
    E, D, F = 2, 32, 16
    recs = [("model.layers.0.mlp.gate.weight", synth(1, E * D, 0.02).reshape(E, D))]
    for e in range(E):
        for proj, rows, cols in (("gate_proj", F, D), ("up_proj", F, D), ("down_proj", D, F)):
            recs.append((f"model.layers.0.mlp.experts.{e}.{proj}.weight", np.zeros((rows, cols), np.float32)))
    p = tmp_path / "f32.bin"
    write_bin(str(p), recs)
    with pytest.raises(mc.MoeError) as ei:
        mc.bin_layer_info(str(p), 0)
    assert ei.value.code == mc.MOE_ERR_UNSUPPORTED


def small_q8(E=4, D=64, F=32):
    L = {"dtype": 2, "router_w": synth(3, E * D, 0.02).reshape(E, D), "router_b": None}
    for nm, (rows, cols) in (("g", (F, D)), ("u", (F, D)), ("d", (D, F))):
        s, q = zip(*[quantize_q8(synth(9 + e, rows * cols, 0.02).reshape(rows, cols)) for e in range(E)])
        L[nm + "s"], L[nm + "q"] = np.stack(s), np.stack(q)
    return L


def test_expert_count_and_shape_checks(tmp_path):
    L = small_q8()
    recs = layer_records(L, 2)
    p = tmp_path / "l.bin"
    write_bin(str(p), recs)
    assert mc.bin_layer_info(str(p), 2) == (4, 64, 32, mc.Q8, 0)
    # experts counted up to the first gap in down_proj (model.h:133-155)
    gap = [r for r in recs if ".experts.2.down_proj" not in r[0]]
    write_bin(str(p), gap)
    with pytest.raises(mc.MoeError):                  # router has 4 rows, 2 experts found
        mc.bin_layer_info(str(p), 2)
    # a missing scale, a wrong shape, a wrong dtype
    for bad in ([r for r in recs if r[0] != "model.layers.2.mlp.experts.1.up_proj.weight.scale"],
                [(n, a[:, :-16] if n.endswith("3.down_proj.weight.q8") else a) for n, a in recs],
                [(n, a.view(np.uint8) if n.endswith("0.up_proj.weight.q8") else a) for n, a in recs]):
        write_bin(str(p), bad)
        with pytest.raises(mc.MoeError) as ei:
            mc.bin_layer_info(str(p), 2)
        assert ei.value.code == mc.MOE_ERR_INVALID


def test_open_handle_find_read():
    with mc.BinFile(REF_BIN) as b:
        # the repeated name resolves to its first record (io.c:333-338)
        assert np.array_equal(b.read("model.norm.weight"), synth(60, 32, 1.0))
        assert b.find("model.layers.3.mlp.experts.2.down_proj.weight.q4") == (3, (32, 8), 256)
        assert b.find("model.layers.3.mlp.router.gate.weight") == (0, (3, 32), 384)
        recs = dict(ref_records()[:4])
        for name, a in recs.items():
            assert np.array_equal(b.read(name), a)
        assert b.layer_info(3) == (3, 32, 16, mc.Q4, 1)
        with pytest.raises(mc.MoeError):
            b.find("model.layers.9.mlp.gate.weight")
        buf = np.empty(31, np.float32)
        assert mc.lib().moe_bin_read(b.h, b"model.norm.weight", buf.ctypes.data, buf.nbytes) == mc.MOE_ERR_INVALID
    with pytest.raises(mc.MoeError):
        mc.BinFile(os.path.join(GOLDEN, "absent.bin"))


def test_host_quantisers_match_exporter():
    """moe_quantize_rowwise_*_host against export._rowwise_q8/_q4 outputs."""
    z = np.load(os.path.join(GOLDEN, "quant.npz"))
    s8, q8 = mc.quantize_rowwise_host(z["W"], mc.Q8)
    s4, q4 = mc.quantize_rowwise_host(z["W"], mc.Q4)
    assert np.array_equal(s8, z["s8"]) and np.array_equal(q8, z["q8"])
    assert np.array_equal(s4, z["s4"]) and np.array_equal(q4, z["q4"])


def test_writer_reproduces_reference_file(tmp_path):
    p = str(tmp_path / "w.bin")
    recs = ref_records()
    w = mc.BinWriter(p, len(recs))
    for name, a in recs:
        w.put(name, a)
    w.finish()
    assert open(p, "rb").read() == open(REF_BIN, "rb").read()


def test_mkbin_matches_reference_export_and_merge(tmp_path):
    """moe_mkbin writes what export.py --outdir + merge_dir.py write for the
    same tensors (tests/golden/mkbin_ref.bin, made by the reference's code)."""
    import subprocess
    tool = os.path.join(os.path.dirname(mc.LIB_PATH), "moe_mkbin")
    p = str(tmp_path / "m.bin")
    subprocess.check_call([tool, "--out", p, "--layers", "2", "--d-model", "64", "--n-q", "4", "--n-kv", "2",
                           "--head-dim", "16", "--d-ff", "32", "--experts", "8", "--vocab", "97", "--seed", "3",
                           "--quant", "q4"])
    assert open(p, "rb").read() == open(os.path.join(GOLDEN, "mkbin_ref.bin"), "rb").read()
    with mc.BinFile(p) as b:
        assert b.layer_info(1) == (8, 64, 32, mc.Q4, 0)
        # header count = original tensors (merge_dir.py:37-39), records beyond it
        assert open(p, "rb").read()[6:10] == (1 + 2 * (9 + 24) + 2).to_bytes(4, "little")


def test_mkbin_record_count_passes_merge_bins(tmp_path):
    """merge_bins.py (the reference's merger of .bin files) reads exactly
    `count` records per input: a file counted by records (--count records)
    passes through it byte for byte, one counted by original tensors (the
    merge_dir.py layout) loses its extra quantised records there."""
    import subprocess
    import sys
    sys.path.insert(0, GOLDEN)
    from make_golden import REF_DIR
    script = os.path.join(REF_DIR, "merge_bins.py")
    if not os.path.exists(script):
        pytest.skip("the reference's merge_bins.py is not present")
    tool = os.path.join(os.path.dirname(mc.LIB_PATH), "moe_mkbin")
    args = ["--layers", "2", "--d-model", "64", "--n-q", "4", "--n-kv", "2", "--head-dim", "16", "--d-ff", "32",
            "--experts", "8", "--vocab", "97", "--seed", "3", "--quant", "q4"]
    for count, whole in (("records", True), ("tensors", False)):
        src, dst = str(tmp_path / f"{count}.bin"), str(tmp_path / f"{count}_merged.bin")
        subprocess.check_call([tool, "--out", src, "--count", count] + args)
        subprocess.check_call([sys.executable, script, dst, src], stdout=subprocess.DEVNULL)
        assert (open(dst, "rb").read() == open(src, "rb").read()) == whole


def test_writer_dtypes_and_errors(tmp_path):
    p = str(tmp_path / "d.bin")
    a16 = np.arange(12, dtype=np.float16).reshape(3, 4)
    scalar = np.array(3.5, np.float32)                   # ndim 0: one element
    w = mc.BinWriter(p, 2)
    w.put("half", a16)
    w.put("scalar", scalar)
    with pytest.raises(mc.MoeError):
        mc.check(mc.lib().moe_bin_put(w.h, b"bad", 7, 0, None, scalar.ctypes.data))   # unknown dtype
    w.finish()
    with mc.BinFile(p) as b:
        assert b.find("half") == (1, (3, 4), 24) and np.array_equal(b.read("half"), a16)
        assert b.find("scalar") == (0, (), 4) and b.read("scalar") == scalar
    assert mc.lib().moe_bin_create(str(tmp_path / "no" / "dir.bin").encode(), 0) is None


def test_corrupted_files_never_crash(tmp_path):
    """Random byte corruptions of the reference-written file (header fields,
    lengths, shapes, data): every call returns a status, and a file that
    still parses keeps the layer's shapes consistent."""
    data = bytearray(open(REF_BIN, "rb").read())
    rng = np.random.default_rng(11)
    p = tmp_path / "fuzz.bin"
    ok = 0
    for trial in range(300):
        d = bytearray(data)
        for _ in range(int(rng.integers(1, 6))):
            pos = int(rng.integers(6, len(d)))
            d[pos] = int(rng.integers(0, 256))
        p.write_bytes(bytes(d))
        try:
            info = mc.bin_layer_info(str(p), 3)
            ok += 1
            assert info[0] == 3 and info[3] == mc.Q4
        except mc.MoeError as e:
            assert e.code in (mc.MOE_ERR_INVALID, mc.MOE_ERR_UNSUPPORTED)
    assert ok > 0
