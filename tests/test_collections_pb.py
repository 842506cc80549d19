"""The protobuf state-dictionary format (engine/ml/src/main/proto/collections.proto) on the host: the reader
against fixtures written by Google's protobuf runtime (tests/golden/make_collections_pb.py), the writer's bytes
against that runtime's serialisation, and StateDictionary(weightsDirectory) semantics of
StateDictionary.loadWeights (engine/ml/src/main/java/org/almostrealism/ml/StateDictionary.java:119-150)."""
import os
import warnings

import numpy as np
import pytest

from common_b200 import Qwen3Config, StateDictionary, collections_pb as P, infer_config, synthetic_state_dict

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _expected():
    e = np.load(os.path.join(GOLDEN, "collections_expected.npz"))
    return {k.replace("__", "."): e[k] for k in e.files}


@pytest.mark.parametrize("name", ["collections_small.pb", "collections_unpacked.pb"])
def test_fixture_decodes(name):
    lib = P.read_library(os.path.join(GOLDEN, name))
    exp = _expected()
    assert set(lib) == set(exp)  # the entry without dimensions is dropped; the repeated key keeps the last
    for k, v in exp.items():
        got = lib[k].numpy()
        assert got.dtype == v.dtype, k
        assert got.shape == v.shape, k
        assert np.array_equal(got, v), k
    assert lib["model.b_f64"].traversal_axis == 1
    assert lib["model.c_3d"].traversal_axis == 2


def _google_classes(packed=True):
    pytest.importorskip("google.protobuf")
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_collections_pb", os.path.join(GOLDEN, "make_collections_pb.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.build_classes(packed, "check_packed.proto" if packed else "check_unpacked.proto")


@pytest.mark.parametrize("precision", ["fp32", "fp64"])
def test_writer_matches_protobuf_runtime(precision):
    cls = _google_classes()
    rng = np.random.default_rng(3)
    w = {"x.weight": rng.standard_normal((3, 5)).astype(np.float32), "y.bias": rng.standard_normal(7),
         "z": np.arange(24, dtype=np.float32).reshape(2, 3, 4), "negative_zero": np.array([-0.0, 1e-30])}
    lib = cls["CollectionLibraryData"]()
    for k, v in w.items():
        e = lib.collections.add()
        e.key = k
        e.collection.traversal_policy.dims.extend(v.shape)
        vals = np.asarray(v, np.float64 if precision == "fp64" else np.float32).ravel().tolist()
        (e.collection.data if precision == "fp64" else e.collection.data_32).extend(vals)
    assert P.encode_library(w, precision) == lib.SerializeToString()
    # and the runtime parses what the writer wrote into the same message
    back = cls["CollectionLibraryData"].FromString(P.encode_library(w, precision))
    assert back == lib


def test_unpacked_reencode_roundtrip(tmp_path):
    """Whatever the protobuf runtime writes unpacked, the reader decodes to the packed file's values."""
    cls_p, cls_u = _google_classes(True), _google_classes(False)
    w = {"a": np.linspace(-1, 1, 12, dtype=np.float32).reshape(3, 4), "b": np.array([np.pi, -np.e])}
    packed = cls_p["CollectionLibraryData"].FromString(P.encode_library(w, "fp32"))
    unpacked = cls_u["CollectionLibraryData"].FromString(packed.SerializeToString())
    raw = unpacked.SerializeToString()
    assert raw != packed.SerializeToString()
    f = tmp_path / "u.pb"
    f.write_bytes(raw)
    lib = P.read_library(str(f))
    for k, v in w.items():
        assert np.array_equal(lib[k].numpy(), v.astype(np.float32))


def test_split_packed_chunks(tmp_path):
    """A repeated field may arrive as several packed chunks; their values concatenate."""
    a = np.arange(6, dtype=np.float32)
    coll = P._len_field(1, P._len_field(1, P._enc_varint(2) + P._enc_varint(3)))
    coll += P._len_field(3, a[:2].tobytes()) + P._len_field(3, a[2:].tobytes())
    raw = P._len_field(1, P._len_field(1, b"k") + P._len_field(2, coll))
    f = tmp_path / "s.pb"
    f.write_bytes(raw)
    assert np.array_equal(P.read_library(str(f))["k"].numpy(), a.reshape(2, 3))


def test_truncated_and_mismatched(tmp_path):
    good = P.encode_library({"a": np.ones((2, 2), np.float32)})
    f = tmp_path / "t.pb"
    f.write_bytes(good[:-3])
    with pytest.raises(P.PbFormatError):
        P.read_library(str(f))
    # 3 values for a (2, 2) shape: the file parses, the tensor does not decode
    coll = P._len_field(1, P._len_field(1, P._enc_varint(2) + P._enc_varint(2)))
    coll += P._len_field(3, np.ones(3, np.float32).tobytes())
    f.write_bytes(P._len_field(1, P._len_field(1, b"a") + P._len_field(2, coll)))
    with pytest.raises(P.PbFormatError):
        P.read_library(str(f))["a"].numpy()


def test_directory_semantics(tmp_path):
    d = tmp_path / "weights"
    d.mkdir()
    P.save({"a": np.full(2, 1, np.float32), "b": np.full(3, 2, np.float32)}, str(d / "00.pb"))
    P.save({"a": np.full(2, 5, np.float32)}, str(d / "01.pb"))  # later files replace keys (name order)
    P.save({"c": np.zeros(1, np.float32)}, str(d / ".hidden.pb"))  # skipped, as StateDictionary skips it
    (d / "02.pb").write_bytes(b"\x0a\xff\xff")  # malformed: warned and skipped
    (d / "sub").mkdir()
    with warnings.catch_warnings(record=True) as w:
        warnings.simplefilter("always")
        sd = StateDictionary(str(d))
    assert any("02.pb" in str(x.message) for x in w)
    assert set(sd.keySet()) == {"a", "b"}
    assert np.array_equal(sd.get("a"), np.full(2, 5, np.float32))
    assert sd.shape("b") == (3,)
    assert not sd.containsKey("c")


@pytest.mark.parametrize("precision", ["fp32", "fp64"])
def test_state_dictionary_save_load_and_infer(tmp_path, precision):
    cfg = Qwen3Config(64, 128, 2, 2, 1, 97, 32, False, headSize=64)
    sd = synthetic_state_dict(cfg, seed=5)
    f = tmp_path / "model.pb"
    sd.save(str(f), precision)
    back = StateDictionary(str(f))
    assert set(back.keySet()) == set(sd.keySet())
    for k in sd.keySet():
        v = back.get(k)
        assert v.dtype == (np.float64 if precision == "fp64" else np.float32)
        assert np.array_equal(v, sd.get(k).astype(v.dtype)), k
    inf = infer_config(back)
    assert (inf.dim, inf.hiddenDim, inf.layerCount, inf.headCount, inf.kvHeadCount, inf.vocabSize, inf.headSize) == \
        (64, 128, 2, 2, 1, 97, 64)
    assert inf.sharedWeights is False
