"""The drop-in claim, checked with the real caller: EB-FaLCom's FalComC.py
(EB-FaLCom/src/appfl/compressor/FalComC.py), unchanged, driving this
library's C ABI.

FalComC loads ``libmomentum_compressor.so`` from its own directory
(FalComC.py:155-178), mirrors the structs in its own ctypes declarations
(:47-105), and compresses / decompresses a model layer by layer through
momentum_compressor_compress_layer / _decompress_layer (:482-679), with its
payloads pickled in between.  Here the file is copied byte for byte from the
reference checkout into a temporary directory next to a copy of a library,
its three imports that are not installed (omegaconf, blosc, APPFL's
BaseCompressor) are stubbed in sys.modules, and the same seeded model rounds
run through:

  * this library's code, built for the host by the kernel emulator (the same
    C host code and the CUDA kernels through the emulator's source
    transform; tests/emu) -- the product library itself needs a GPU;
  * the reference's own codec (oracle/_ref).

With the raw residual codec and libzstd frames every pickled layer (all
fields but the wall-clock breakdown timers) and every decoded layer is
identical between the two, and each decoder reads the other's payloads; in
the default q8 mode FalComC's round trip works and decodes within the q8
quality bar of the reference's own GPU codec tests (rel-L2 <= 0.02,
cuda_feasibility/falcom_cuda_v4/tests/test_cuda_v4_codec_quality.py:30-60).

The reference checkout is read only here, in this container (the test skips
without it); the GPU box never reads it."""
import importlib.util
import os
import pickle
import shutil
import sys
import types
from collections import OrderedDict

import numpy as np
import pytest

from oracle import binding as ob
from oracle.reference_root import reference_root

torch = pytest.importorskip("torch")

FALCOMC = os.path.join("EB-FaLCom", "src", "appfl", "compressor", "FalComC.py")
SHAPES = [("conv1.weight", (16, 3, 3, 3)), ("bn1.weight", (16,)), ("bn1.bias", (16,)),
          ("bn1.running_mean", (16,)), ("bn1.running_var", (16,)), ("bn1.num_batches_tracked", ()),
          ("layer1.0.conv1.weight", (32, 16, 3, 3)), ("layer1.0.conv2.weight", (64, 32, 1, 1)),
          ("layer1.0.bn1.weight", (32,)), ("fc.weight", (10, 256)), ("fc.bias", (10,))]


class _Config:
    """The attributes and get() FalComC reads from its DictConfig (:220-253);
    lossless_compressor is left unset, so FalComC picks its own default."""

    def __init__(self, **kw):
        self.__dict__.update(kw)

    def get(self, key, default=None):
        return self.__dict__.get(key, default)


def _stub_modules(monkeypatch):
    omegaconf = types.ModuleType("omegaconf")
    omegaconf.DictConfig = dict
    monkeypatch.setitem(sys.modules, "omegaconf", omegaconf)
    monkeypatch.setitem(sys.modules, "blosc", types.ModuleType("blosc"))
    base = types.ModuleType("appfl.compressor.base_compressor")

    class BaseCompressor:
        def __init__(self, compressor_config):
            pass
    base.BaseCompressor = BaseCompressor
    for name in ("appfl", "appfl.compressor"):
        monkeypatch.setitem(sys.modules, name, types.ModuleType(name))
    monkeypatch.setitem(sys.modules, "appfl.compressor.base_compressor", base)


def _falcomc_with(lib_path, where, tag):
    """FalComC.py, byte for byte, in `where` beside a copy of `lib_path`
    named libmomentum_compressor.so; the module is imported from there."""
    os.makedirs(where, exist_ok=True)
    shutil.copyfile(os.path.join(reference_root(), FALCOMC), os.path.join(where, "FalComC.py"))
    shutil.copyfile(lib_path, os.path.join(where, "libmomentum_compressor.so"))
    spec = importlib.util.spec_from_file_location(f"falcomc_{tag}", os.path.join(where, "FalComC.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _rounds(n_rounds, seed=17):
    rng = np.random.default_rng(seed)
    state = {}
    out = []
    for t in range(n_rounds):
        model = OrderedDict()
        for name, shape in SHAPES:
            if name.endswith("num_batches_tracked"):
                model[name] = torch.tensor(100 * (t + 1), dtype=torch.int64)
                continue
            fan = int(np.prod(shape[1:])) if len(shape) >= 2 else shape[0]
            noise = rng.standard_normal(shape) * (1e-3 / np.sqrt(fan))
            state[name] = noise if t == 0 else 0.9 * state[name] + noise
            model[name] = torch.from_numpy(state[name].astype(np.float32))
        out.append(model)
    return out


def _strip(layers):
    return {k: ({f: v for f, v in d.items() if not f.startswith("breakdown_")} if isinstance(d, dict) else d)
            for k, d in layers.items()}


@pytest.fixture(scope="module")
def emu_lib():
    from tests.emu import build as emu_build
    return emu_build.build()


@pytest.fixture()
def falcomc_env(monkeypatch, tmp_path):
    if not reference_root() or not os.path.exists(os.path.join(reference_root(), FALCOMC)):
        pytest.skip("reference checkout (EB-FaLCom/.../FalComC.py) not present")
    _stub_modules(monkeypatch)
    monkeypatch.chdir(tmp_path)          # FalComC writes ./output/falcom_c.log
    monkeypatch.setenv("FALCOM_LOG_LEVEL", "ERROR")
    return tmp_path


def _run(mod, rounds, cfg):
    enc = mod.FalComC(cfg)
    dec = mod.FalComC(cfg)
    blobs, decoded = [], []
    for model in rounds:
        blob = enc.compress_model(model, client_id="Client1")
        blobs.append(blob)
        decoded.append(dec.decompress_model(blob, client_id="Client1"))
    return enc, dec, blobs, decoded


def test_falcomc_unchanged_raw_mode_identical_to_reference(falcomc_env, emu_lib, monkeypatch):
    if not ob.have_ref():
        pytest.skip("reference build oracle/_ref not present")
    monkeypatch.setenv("FALCOM_RESIDUAL_CODEC", "raw")
    monkeypatch.setenv("FALCOM_FRAME_MODE", "libzstd")
    ours = _falcomc_with(emu_lib, str(falcomc_env / "ours"), "ours")
    ref = _falcomc_with(ob.REF_SO, str(falcomc_env / "ref"), "ref")
    rounds = _rounds(4)
    cfg = _Config(momentum_lr=0.07, consistency_threshold=0.5, param_cutoff=1024,
                  sz_config={"error_bounding_mode": "REL", "error_bound": 1e-3})
    _, _, blobs_a, dec_a = _run(ours, rounds, cfg)
    _, _, blobs_b, dec_b = _run(ref, rounds, cfg)
    kinds = set()
    for t, (ba, bb) in enumerate(zip(blobs_a, blobs_b)):
        la, lb = pickle.loads(ba), pickle.loads(bb)
        assert list(la) == list(lb)
        assert _strip(la) == _strip(lb), t
        kinds |= {d.get("c_type", d["codec"]) for d in la.values()}
    # (the 0-dim counter reaches C as one element: np.ascontiguousarray in
    # FalComC.py:273 returns at least one dimension)
    assert {"direct", "direct_generic", "momentum_predicted"} <= kinds
    for da, db in zip(dec_a, dec_b):
        for name in da:
            a, b = da[name].numpy(), db[name].numpy()
            assert a.dtype == b.dtype and a.shape == b.shape, name
            assert np.array_equal(a.view(np.uint8), b.view(np.uint8)), name
    # each decoder reads the other's payloads
    cross_a = ours.FalComC(cfg)
    cross_b = ref.FalComC(cfg)
    for ba, bb, da in zip(blobs_a, blobs_b, dec_a):
        xa = cross_a.decompress_model(bb, client_id="Client1")
        xb = cross_b.decompress_model(ba, client_id="Client1")
        for name in da:
            assert np.array_equal(xa[name].numpy().view(np.uint8), da[name].numpy().view(np.uint8)), name
            assert np.array_equal(xb[name].numpy().view(np.uint8), da[name].numpy().view(np.uint8)), name


def test_falcomc_unchanged_default_q8_round_trip(falcomc_env, emu_lib, monkeypatch):
    monkeypatch.delenv("FALCOM_RESIDUAL_CODEC", raising=False)
    monkeypatch.delenv("FALCOM_FRAME_MODE", raising=False)
    ours = _falcomc_with(emu_lib, str(falcomc_env / "ours_q8"), "ours_q8")
    rounds = _rounds(4, seed=5)
    cfg = _Config(momentum_lr=0.07, consistency_threshold=0.5, param_cutoff=1024,
                  sz_config={"error_bounding_mode": "REL", "error_bound": 1e-3})
    _, _, blobs, decoded = _run(ours, rounds, cfg)
    n_pred = 0
    for model, blob, out in zip(rounds, blobs, decoded):
        layers = pickle.loads(blob)
        assert list(out) == list(model)
        for name, x in model.items():
            d = layers[name]
            y = out[name]
            if d["codec"] == "pickle":
                assert torch.equal(y, x)
                continue
            n_pred += d["c_type"] == "momentum_predicted"
            if d["c_codec"] == "q8":
                a, b = x.numpy().astype(np.float64).ravel(), y.numpy().astype(np.float64).ravel()
                assert np.linalg.norm(a - b) <= 0.02 * np.linalg.norm(a), name
            else:
                # lossless (a 0-dim counter comes back with the one
                # dimension it crossed the C ABI with)
                assert torch.equal(y.reshape(x.shape), x), name
    assert n_pred > 0
