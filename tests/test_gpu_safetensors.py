"""Checkpoint interoperability of zrl_save / zrl_load_from_bytes with the
safetensors format that ActorCritic::save writes (ppo.rs:529-575) and
load_from_bytes reads (ppo.rs:585-650).

The reference serializes with the Rust safetensors crate (no metadata, every
tensor F32); the Python `safetensors` package in this image wraps the same
Rust serializer, so it stands in for the reference's writer and reader:
* its loader reads our file with the reference's tensor names, shapes and
  dtype, and the values we hold;
* its writer, given the same tensors, produces our file byte for byte;
* a file it writes loads through zrl_load_from_bytes with every value intact.
"""
import numpy as np
import pytest

from zealot_b200 import zealot_rl as Z

pytestmark = pytest.mark.gpu

safetensors_numpy = pytest.importorskip("safetensors.numpy")

ADIMS, CDIMS = (12, 64, 32, 5), (10, 64, 32, 1)


def _reference_tensors(ac):
    """The tensors ActorCritic::save pushes, by name (ppo.rs:539-571)."""
    flat = ac.params
    out, off = {}, 0
    for prefix, dims in (("actor", ADIMS), ("critic", CDIMS)):
        for l in range(len(dims) - 1):
            fi, fo = dims[l], dims[l + 1]
            out[f"{prefix}.w_{l}"] = flat[off:off + fo * fi].reshape(fo, fi)
            off += fo * fi
            out[f"{prefix}.b_{l}"] = flat[off:off + fo]
            off += fo
    out["log_std"] = flat[off:]
    om, om2, oc, cm, cm2, cc = ac.normalizers()
    out["obs_norm.mean"], out["obs_norm.m2"] = om, om2
    out["obs_norm.count"] = np.array([oc], np.float32)
    out["critic_norm.mean"], out["critic_norm.m2"] = cm, cm2
    out["critic_norm.count"] = np.array([cc], np.float32)
    out["lr"] = np.array([ac.lr], np.float32)
    return out


@pytest.fixture
def trained(tmp_path):
    rng = Z.Lcg(11)
    ac = Z.ActorCritic.new(ADIMS, CDIMS, 0.7, 2e-3, rng, precision="fp32")
    g = np.random.default_rng(5)
    ac.record_obs(g.standard_normal((40, ADIMS[0]), dtype=np.float32) * 2 + 1,
                  g.standard_normal((40, CDIMS[0]), dtype=np.float32))
    path = str(tmp_path / "policy.safetensors")
    ac.save(path)
    return ac, path


def test_reference_reader_sees_the_reference_layout(trained):
    ac, path = trained
    got = safetensors_numpy.load_file(path)
    want = _reference_tensors(ac)
    assert sorted(got) == sorted(want)
    for name, arr in want.items():
        assert got[name].dtype == np.float32, name
        assert got[name].shape == arr.shape, name
        assert np.array_equal(got[name], arr), name


def test_file_equals_the_reference_writer_byte_for_byte(trained, tmp_path):
    ac, path = trained
    ref = str(tmp_path / "ref.safetensors")
    safetensors_numpy.save_file({k: np.ascontiguousarray(v) for k, v in
                                 _reference_tensors(ac).items()}, ref)
    assert open(path, "rb").read() == open(ref, "rb").read()


def test_reference_written_file_loads(trained, tmp_path):
    ac, _ = trained
    tensors = _reference_tensors(ac)
    g = np.random.default_rng(9)
    tensors = {k: (v + g.standard_normal(v.shape).astype(np.float32) * 0.01
                   if k.startswith(("actor", "critic.")) else v) for k, v in tensors.items()}
    ref = str(tmp_path / "ref.safetensors")
    safetensors_numpy.save_file({k: np.ascontiguousarray(v) for k, v in tensors.items()}, ref)
    ac2 = Z.ActorCritic.load_from_bytes(open(ref, "rb").read(), precision="fp32")
    back = _reference_tensors(ac2)
    for name, arr in tensors.items():
        assert np.array_equal(back[name], arr), name
