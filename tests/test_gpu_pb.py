"""Weights from the reference's protobuf state-dictionary files through the library's own loader
(qw_load_state_dict_pb): the same device weights, bit for bit, as loading the arrays one by one, and greedy
generation equal to the oracle's, through StateDictionary(weightsDirectory) and Qwen3."""
import os

import numpy as np
import pytest

from common_b200 import Qwen3, Qwen3Config, StateDictionary, collections_pb as P, native
from tests.helpers import cfg_dict, native_model, oracle_model, state_dict

pytestmark = pytest.mark.gpu


def _empty_model(c, precision="fp32"):
    dt = {"fp32": native.DTYPE_F32, "bf16": native.DTYPE_BF16}[precision]
    cfg = native.make_config(c["dim"], c["hidden_dim"], c["layers"], c["heads"], c["kv_heads"], c["head_dim"],
                             c["vocab"], c["seq_len"], c["shared_weights"], c["qk_norm"], c["has_qkv_bias"], dt, dt, 1,
                             0, 64, 0, c["rope_theta"], c["eps"], 0)
    return native.NativeModel(cfg, 0)


def _logits(m, toks):
    out = []
    for i, t in enumerate(toks):
        lg, _ = m.decode_step([int(t)], [i])
        out.append(lg[0].copy())
    return np.stack(out)


def _write_split(sd, d):
    """The state dict over three files (fp32, fp64 and fp32), plus files the loader must pass over."""
    keys = list(sd)
    third = len(keys) // 3
    P.save({k: sd[k] for k in keys[:third]}, os.path.join(d, "a.pb"), "fp32")
    P.save({k: sd[k] for k in keys[third:2 * third]}, os.path.join(d, "b.pb"), "fp64")
    P.save({k: sd[k] for k in keys[2 * third:]}, os.path.join(d, "c.pb"), "fp32")
    P.save({"model.norm.weight": np.zeros(3, np.float32)}, os.path.join(d, ".ignored.pb"))
    P.save({"model.rotary_emb.inv_freq": np.ones(32, np.float32)}, os.path.join(d, "d_unused.pb"))
    with open(os.path.join(d, "e_broken.pb"), "wb") as f:
        f.write(b"\x0a\x80")


@pytest.mark.parametrize("precision", ["fp32", "bf16"])
def test_pb_directory_equals_tensor_loads(tmp_path, precision):
    c = cfg_dict(seq_len=40)
    sd = state_dict(c, seed=31, std=0.05)
    _write_split(sd, str(tmp_path))
    m = _empty_model(c, precision)
    n = m.load_state_dict_pb(str(tmp_path))
    assert n == len(sd)
    assert "e_broken.pb" in native.load().qw_last_error(m.h).decode()
    m.finalize()
    ref = native_model(c, sd, precision=precision)
    toks = np.random.default_rng(32).integers(0, c["vocab"], 24)
    a, b = _logits(m, toks), _logits(ref, toks)
    assert np.array_equal(a, b)  # fp64 values of the same fp32 numbers convert to the same device weights
    m.close()
    ref.close()


def test_pb_unpacked_file(tmp_path):
    """A file written with every repeated scalar unpacked loads to the same weights."""
    pytest.importorskip("google.protobuf")
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "make_collections_pb", os.path.join(os.path.dirname(__file__), "golden", "make_collections_pb.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    cls_p, cls_u = mod.build_classes(True, "gpu_packed.proto"), mod.build_classes(False, "gpu_unpacked.proto")
    c = cfg_dict(layers=1, seq_len=16)
    sd = state_dict(c, seed=33, std=0.05)
    packed = cls_p["CollectionLibraryData"].FromString(P.encode_library(sd, "fp32"))
    (tmp_path / "u.pb").write_bytes(cls_u["CollectionLibraryData"].FromString(packed.SerializeToString())
                                    .SerializeToString())
    m = _empty_model(c)
    assert m.load_state_dict_pb(str(tmp_path / "u.pb")) == len(sd)
    m.finalize()
    ref = native_model(c, sd)
    toks = [5, 9, 2, 7]
    assert np.array_equal(_logits(m, toks), _logits(ref, toks))
    m.close()
    ref.close()


def test_pb_shape_error_and_missing_path(tmp_path):
    c = cfg_dict(layers=1, seq_len=16)
    m = _empty_model(c)
    P.save({"model.norm.weight": np.zeros(c["dim"] + 1, np.float32)}, str(tmp_path / "bad.pb"))
    with pytest.raises(native.QwenError) as e:
        m.load_state_dict_pb(str(tmp_path / "bad.pb"))
    assert e.value.status == 2  # QW_ERR_SHAPE from qw_load_tensor
    with pytest.raises(native.QwenError):
        m.load_state_dict_pb(str(tmp_path / "nope"))
    m.close()


def test_qwen3_from_weights_directory(tmp_path):
    """Qwen3(config, StateDictionary(weightsDirectory)) generates what the oracle generates."""
    c = cfg_dict(seq_len=32)
    sd = state_dict(c, seed=34, std=0.08)
    P.save(sd, str(tmp_path / "weights.pb"))
    cfg = Qwen3Config(c["dim"], c["hidden_dim"], c["layers"], c["heads"], c["kv_heads"], c["vocab"], 32, False,
                      headSize=c["head_dim"])
    q = Qwen3(cfg, StateDictionary(str(tmp_path)), precision="fp32")
    got = q.generate([3, 1, 4], 16)[0]
    want, _ = oracle_model(c, sd).generate(np.array([3, 1, 4], np.int32), 16)
    assert list(got) == list(want)
    q.close()
