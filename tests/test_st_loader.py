"""The safetensors readers, CPU only: the expert-run loader (k3_bank_read_safetensors) and
the tensor index over a shard set (k3_st_open / find / read, any tensor by name).

Shards are written here in the checkpoint format the reference documents (src/io/k3_st.h:
7-13: 8-byte little-endian header length, JSON header, data with offsets relative to the
header's end) with the expert tensor names of src/io/k3_load.c:11, and the awkward header
cases a hand-written scanner gets wrong (escaped names, __metadata__, a scalar shape, a
zero-element tensor, other dtypes). The bank bytes must be the tensors exactly, in the
run order w1.packed w1.scale w2.packed w2.scale w3.packed w3.scale (src/io/k3_load.h:1-22).
"""
import json
import os
import struct
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from k3lib import load  # noqa: E402

L, I, LAYER = 64, 96, 3
NAME = "language_model.model.layers.{}.block_sparse_moe.experts.{}.{}.{}"


@pytest.fixture(scope="module")
def k3():
    return load()


def expert_tensors(rng, e):
    t = {}
    for w, rows, cols in (("w1", I, L), ("w2", L, I), ("w3", I, L)):
        t[(w, "weight_packed")] = rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
        t[(w, "weight_scale")] = rng.integers(0, 256, (rows, cols // 32), dtype=np.uint8)
    return t


def write_shard(path, tensors, metadata=None, order=None):
    """tensors: name -> (dtype string, shape list, raw bytes)."""
    names = order or list(tensors)
    header, blobs, off = {}, [], 0
    if metadata is not None:
        header["__metadata__"] = metadata
    for n in names:
        dt, shape, raw = tensors[n]
        header[n] = {"dtype": dt, "shape": shape, "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header, ensure_ascii=True).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def u8(a):
    return ("U8", list(a.shape), a.tobytes())


def build_shards(tmp_path, rng, n_exp=4):
    ex = [expert_tensors(rng, e) for e in range(n_exp)]
    a, b = {}, {}
    for e in range(n_exp):
        dst = a if e < 2 else b
        for (w, kind), arr in ex[e].items():
            dst[NAME.format(LAYER, e, w, kind)] = u8(arr)
    # other tensors and awkward entries in shard A
    a["language_model.model.layers.3.input_layernorm.weight"] = ("BF16", [L], np.zeros(L, np.uint16).tobytes())
    a['odd "name" with \\ escapes and é'] = ("F32", [], np.float32(1.5).tobytes())
    a["an.empty.tensor"] = ("F16", [0, 7], b"")
    # shard B stores expert 3's tensors in reversed order (not one contiguous run)
    order_b = [k for k in b if ".experts.2." in k] + list(reversed([k for k in b if ".experts.3." in k]))
    pa, pb = str(tmp_path / "model-00001-of-00002.safetensors"), str(tmp_path / "model-00002-of-00002.safetensors")
    write_shard(pa, a, metadata={"format": "pt", "note": "escapes \" \\ / \n"})
    write_shard(pb, b, order=order_b)
    return ex, [pb, pa]                                  # any order


def check_run(k3, run, tens):
    lay = k3.ExpertBank.layout(L, I)
    for (w, kind), arr in tens.items():
        off = {("w1", "weight_packed"): lay.p1, ("w1", "weight_scale"): lay.s1,
               ("w2", "weight_packed"): lay.p2, ("w2", "weight_scale"): lay.s2,
               ("w3", "weight_packed"): lay.p3, ("w3", "weight_scale"): lay.s3}[(w, kind)]
        np.testing.assert_array_equal(run[off:off + arr.size], arr.reshape(-1))


def test_run_order_is_the_checkpoint_order(k3):
    lay = k3.ExpertBank.layout(L, I)
    offs = [lay.p1, lay.s1, lay.p2, lay.s2, lay.p3, lay.s3]
    sizes = [I * L // 2, I * L // 32, L * I // 2, L * I // 32, I * L // 2, I * L // 32]
    assert offs == sorted(offs) and offs[0] == 0
    assert all(offs[i] + sizes[i] <= offs[i + 1] for i in range(5)) and offs[5] + sizes[5] <= lay.stride


def test_reads_experts_across_shards(k3, tmp_path):
    ex, files = build_shards(tmp_path, np.random.default_rng(1))
    lay = k3.ExpertBank.layout(L, I)
    buf = k3.bank_read_safetensors(files, LAYER, 1, 3, L, I)    # experts 1, 2, 3
    assert buf.size == 3 * lay.stride
    for j, e in enumerate((1, 2, 3)):
        check_run(k3, buf[j * lay.stride:(j + 1) * lay.stride], ex[e])


def test_errors(k3, tmp_path):
    ex, files = build_shards(tmp_path, np.random.default_rng(2))
    lay = k3.ExpertBank.layout(L, I)
    lib = k3.lib
    C = k3.C
    arr = (C.c_char_p * 2)(*[os.fsencode(f) for f in files])
    buf = np.zeros(4 * lay.stride, np.uint8)
    # an expert that is not there, a layer that is not there
    assert lib.k3_bank_read_safetensors(arr, 2, LAYER, 3, 2, L, I, buf.ctypes.data, buf.nbytes) == k3.K3GPU_EINVAL
    assert lib.k3_bank_read_safetensors(arr, 2, LAYER + 1, 0, 1, L, I, buf.ctypes.data, buf.nbytes) == k3.K3GPU_EINVAL
    # too small a buffer
    assert lib.k3_bank_read_safetensors(arr, 2, LAYER, 0, 4, L, I, buf.ctypes.data, 3 * lay.stride) == \
        k3.K3GPU_ECAPACITY
    # wrong geometry: the tensors are [I][L/2], not [L][I/2]
    assert lib.k3_bank_read_safetensors(arr, 2, LAYER, 0, 1, I, L, buf.ctypes.data, buf.nbytes) == k3.K3GPU_EINVAL
    # a wrong dtype, data past the end of the file, a malformed header
    t = expert_tensors(np.random.default_rng(3), 0)
    bad = {NAME.format(LAYER, 0, w, kind): u8(a) for (w, kind), a in t.items()}
    key = NAME.format(LAYER, 0, "w2", "weight_scale")
    bad[key] = ("I8",) + bad[key][1:]
    p = str(tmp_path / "bad_dtype.safetensors")
    write_shard(p, bad)
    one = (C.c_char_p * 1)(os.fsencode(p))
    assert lib.k3_bank_read_safetensors(one, 1, LAYER, 0, 1, L, I, buf.ctypes.data, buf.nbytes) == k3.K3GPU_EINVAL
    good = {NAME.format(LAYER, 0, w, kind): u8(a) for (w, kind), a in t.items()}
    p = str(tmp_path / "short.safetensors")
    write_shard(p, good)
    with open(p, "r+b") as f:
        f.truncate(os.path.getsize(p) - 10)
    one = (C.c_char_p * 1)(os.fsencode(p))
    assert lib.k3_bank_read_safetensors(one, 1, LAYER, 0, 1, L, I, buf.ctypes.data, buf.nbytes) == k3.K3GPU_EINVAL
    p = str(tmp_path / "junk.safetensors")
    with open(p, "wb") as f:
        h = b'{"a": {"dtype": "U8", "shape": [1], "data_offsets": [0, 1]'
        f.write(struct.pack("<Q", len(h)) + h + b"\0")
    one = (C.c_char_p * 1)(os.fsencode(p))
    assert lib.k3_bank_read_safetensors(one, 1, LAYER, 0, 1, L, I, buf.ctypes.data, buf.nbytes) == k3.K3GPU_EINVAL
    missing = (C.c_char_p * 1)(os.fsencode(str(tmp_path / "absent.safetensors")))
    assert lib.k3_bank_read_safetensors(missing, 1, LAYER, 0, 1, L, I, buf.ctypes.data, buf.nbytes) == k3.K3GPU_EINVAL
    # offsets near the top of the 64-bit range (a sum that would wrap), an expert range
    # whose end would wrap an int
    p = str(tmp_path / "huge.safetensors")
    with open(p, "wb") as f:
        h = b'{"a": {"dtype": "U8", "shape": [1], "data_offsets": [9223372036854775000, 9223372036854775807]}}'
        f.write(struct.pack("<Q", len(h)) + h + b"\0")
    one = (C.c_char_p * 1)(os.fsencode(p))
    assert lib.k3_bank_read_safetensors(one, 1, LAYER, 0, 1, L, I, buf.ctypes.data, buf.nbytes) == k3.K3GPU_EINVAL
    assert lib.k3_bank_read_safetensors(arr, 2, LAYER, 2 ** 31 - 2, 4, L, I, buf.ctypes.data, buf.nbytes) == \
        k3.K3GPU_EINVAL


def test_tensor_index_reads_any_tensor(k3, tmp_path):
    """k3_st_open / find / read: every tensor of both shards by name (escaped names, bf16,
    f32, f16, u8, an empty tensor), in discovery order, opened by directory or by paths;
    the expert tensors read through it equal what the expert-run reader placed."""
    rng = np.random.default_rng(7)
    ex, files = build_shards(tmp_path, rng)
    trunk = rng.standard_normal((5, 12)).astype(np.float32)
    bf = (rng.standard_normal(33).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    extra = {"language_model.model.embed_tokens.weight": ("F32", [5, 12], trunk.tobytes()),
             "language_model.model.norm.weight": ("BF16", [33], bf.tobytes()),
             "unicode.é€.name": ("I64", [2], np.arange(2, dtype=np.int64).tobytes())}
    pc = str(tmp_path / "model-00003-of-00003.safetensors")
    write_shard(pc, extra)
    for where in (str(tmp_path), files + [pc]):
        idx = k3.SafetensorsIndex(where)
        names = idx.names()
        assert len(names) == len(set(names)) == 4 * 6 + 3 + 3
        e = idx.info("language_model.model.embed_tokens.weight")
        assert (e["dtype"], e["shape"], e["nbytes"]) == (k3.ST_F32, [5, 12], trunk.nbytes)
        np.testing.assert_array_equal(idx.read("language_model.model.embed_tokens.weight"), trunk)
        np.testing.assert_array_equal(idx.read("language_model.model.norm.weight"), bf)
        assert idx.info('odd "name" with \\ escapes and é')["shape"] == []
        assert idx.read('odd "name" with \\ escapes and é').tobytes() == np.float32(1.5).tobytes()
        assert idx.info("an.empty.tensor")["nbytes"] == 0
        u = idx.info("unicode.é€.name")
        assert (u["dtype"], u["dtype_name"]) == (k3.ST_UNKNOWN, "I64")
        for e_ in range(4):
            for (w, kind), arr in ex[e_].items():
                got = idx.read(NAME.format(LAYER, e_, w, kind))
                assert got.dtype == np.uint8 and got.shape == arr.shape
                np.testing.assert_array_equal(got, arr)
        with pytest.raises(k3.K3Error):
            idx.info("no.such.tensor")
        C = k3.C
        small = np.empty(10, np.uint8)
        assert k3.lib.k3_st_read(idx._s, b"language_model.model.embed_tokens.weight", small.ctypes.data,
                                 small.nbytes) == k3.K3GPU_ECAPACITY
        idx.close()
    # the directory form visits shards by name: shard 1 first, in header order
    idx = k3.SafetensorsIndex(str(tmp_path))
    assert idx.info(idx.names()[0])["shard"] == 0
    assert idx.names()[-1] == "unicode.é€.name"
    idx.close()


def test_tensor_index_refuses_broken_sets(k3, tmp_path):
    rng = np.random.default_rng(8)
    ok = tmp_path / "ok"
    ok.mkdir()
    ex, files = build_shards(ok, rng)
    dup = str(tmp_path / "dup.safetensors")
    write_shard(dup, {NAME.format(LAYER, 0, "w1", "weight_scale"): u8(ex[0][("w1", "weight_scale")])})
    with pytest.raises(k3.K3Error):
        k3.SafetensorsIndex(files + [dup])                 # a name in two shards
    short = str(tmp_path / "short.safetensors")
    write_shard(short, {"t": ("F32", [4], np.zeros(4, np.float32).tobytes())})
    with open(short, "r+b") as f:
        f.truncate(os.path.getsize(short) - 4)
    with pytest.raises(k3.K3Error):
        k3.SafetensorsIndex([short])                       # data past the end
    with pytest.raises(k3.K3Error):
        k3.SafetensorsIndex(str(tmp_path / "empty_dir_that_does_not_exist"))


def test_deeply_nested_header_is_refused_not_overflowed(k3, tmp_path):
    """A header whose metadata nests arrays far deeper than any checkpoint (a crafted or
    corrupt shard) is refused as malformed; nesting within the bound still reads."""
    import json
    import struct

    def shard(path, depth):
        meta = "[" * depth + "1" + "]" * depth
        body = json.dumps({"t": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]}})
        hdr = ('{"__metadata__": {"x": %s}, %s' % (meta, body[1:])).encode()
        with open(path, "wb") as f:
            f.write(struct.pack("<Q", len(hdr)))
            f.write(hdr)
            f.write(np.arange(2, dtype=np.float32).tobytes())
        return str(path)

    ok = shard(tmp_path / "ok.safetensors", 40)
    idx = k3.SafetensorsIndex([ok])
    assert idx.read("t").view(np.float32).tolist() == [0.0, 1.0]
    idx.close()
    bad = shard(tmp_path / "deep.safetensors", 200000)
    with pytest.raises(k3.K3Error):
        k3.SafetensorsIndex([bad])
