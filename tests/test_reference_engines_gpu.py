"""The drop-ins running inside the reference's own engines.

The unmodified reference package (streamtrain, morph) is installed into
baseline/_ref by ``__graft_entry__.build()``; these tests import it from there,
apply the patches a MORPH maintainer would apply (the drop-in classes swapped
in by name, ``morph_b200.disk_io.patch_class`` / ``patch_cached_class`` on the
store classes, the device ``DynamicLossScale`` behind
``streamtrain.precision.DynamicLossScale``), and run the reference's own
hot-path scenarios next to the unpatched reference on identical inputs:

* tests/test_training.py:9-27 (MORPH paths): the Hybrid optimizer's AdamW
  group equals torch AdamW bit for bit over three steps, and a NaN gradient
  raises FloatingPointError with the model unchanged; :50-64, the Muon
  diagonal known answer (held to the 1e-2 Muon tolerance of 16-bit
  Newton-Schulz, not the FP32 reference's 1e-5);
* tests/test_fp16.py:59-72: the real ``DiskDLS.step`` overflow loop on FP16
  compute, loss scales [128, 64] in order and 64 persisted in the manifest;
  :41-50, a fault in the middle of the state write, then ``resume_step``, gives
  the files of a clean step;
* tests/test_sparse_disk.py:16-38 and :40-58: ``SparseDiskDLS`` against
  clip_grad_norm_ + torch AdamW (conditional clocks, inactive experts
  untouched), and its fault-and-resume recovery, byte for byte;
* tests/test_state_cache.py:34-46: ``CachedDiskState`` hits through
  ``patch_cached_class``, byte-identical to the plain store;
* morph/training/runner.py:46,100-101: the resident training loop with the
  drop-in AdamW behind torch.optim.AdamW (clip_grad_norm_ then step), close to
  the unpatched run and bit-identical across a checkpoint and resume.

Cross-implementation comparisons use the reference's own tolerances; the two
store paths of one implementation are compared byte for byte.
"""
import copy
import os
import sys
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(REPO, "baseline", "_ref")


@pytest.fixture(scope="module")
def ref():
    if not os.path.isdir(os.path.join(REF, "streamtrain")):
        pytest.fail("the reference is not installed in baseline/_ref: run __graft_entry__.build() "
                    "where the reference checkout is present")
    if REF not in sys.path:
        sys.path.insert(0, REF)
    import morph
    import streamtrain
    for mod in (streamtrain, morph):
        assert os.path.realpath(mod.__file__).startswith(os.path.realpath(REF)), mod.__file__
    return REF


def _patch_loss_scale(mp):
    """DiskDLS.__init__ imports DynamicLossScale from streamtrain.precision at
    call time (streamtrain/disk.py:243-244): swap the device one in by name."""
    import streamtrain.precision
    import morph_b200
    mp.setattr(streamtrain.precision, "DynamicLossScale",
               lambda scale=128., growth_interval=2000: morph_b200.DynamicLossScale(scale, growth_interval,
                                                                                    device="cuda"))


def _patch_stores(mp, cached=False):
    """Every DiskState (and CachedDiskState) instance's update() on the GPU."""
    import streamtrain.disk
    import streamtrain.state_cache
    from morph_b200.disk_io import patch_cached_class, patch_class
    restore = [patch_class(streamtrain.disk.DiskState, "cuda")]
    if cached:
        restore.append(patch_cached_class(streamtrain.state_cache.CachedDiskState, "cuda"))
    return restore


class _Patched:
    """Apply the store / loss-scale patches for the duration of a with block."""

    def __init__(self, stores=True, cached=False, loss_scale=True):
        self.stores, self.cached, self.loss_scale = stores, cached, loss_scale
        self.mp = pytest.MonkeyPatch()
        self.restore = []

    def __enter__(self):
        if self.loss_scale:
            _patch_loss_scale(self.mp)
        if self.stores:
            self.restore = _patch_stores(self.mp, self.cached)
        return self

    def __exit__(self, *exc):
        for r in reversed(self.restore):
            r()
        self.mp.undo()


def _entry_planes(store, name):
    entry = store.entries[name]
    return np.fromfile(os.path.join(str(store.root), entry["file"]), dtype=np.float32).reshape(3, entry["size"])


# -------------------------------------------- tests/test_training.py:9-64 --

def _tiny_morph():
    from morph import MorphConfig, MorphModel
    return MorphModel(MorphConfig(vocab_size=16, d_model=8, num_layers=1, d_ff=16, d_state=2, head_dim=4))


def test_hybrid_adam_group_matches_torch_and_nan_is_atomic(ref, cuda, monkeypatch):
    import morph_b200
    import streamtrain.optimizer
    monkeypatch.setattr(streamtrain.optimizer, "HybridMuonAdamW", morph_b200.HybridMuonAdamW)
    torch.manual_seed(0)
    model = _tiny_morph()
    _, auxiliary = streamtrain.optimizer.partition(model)
    reference = [torch.nn.Parameter(p.detach().clone()) for p in auxiliary]  # torch AdamW on the CPU
    model = model.to(cuda)
    _, auxiliary = streamtrain.optimizer.partition(model)
    hybrid = streamtrain.optimizer.HybridMuonAdamW(model, lr=.003)
    assert isinstance(hybrid, morph_b200.HybridMuonAdamW)
    adam = torch.optim.AdamW(reference, lr=.003, weight_decay=.01, betas=(.9, .95), foreach=False)
    for _ in range(3):
        for p, q in zip(auxiliary, reference):
            p.grad = torch.ones_like(p) * .2
            q.grad = p.grad.cpu().clone()
        hybrid.step()
        adam.step()
    for p, q in zip(auxiliary, reference):
        torch.testing.assert_close(p.detach().cpu(), q.detach(), rtol=0, atol=0)
    before = copy.deepcopy(model.state_dict())
    next(model.parameters()).grad.fill_(float("nan"))
    with pytest.raises(FloatingPointError):
        hybrid.step()
    for key, value in model.state_dict().items():
        torch.testing.assert_close(value, before[key], rtol=0, atol=0)


def test_muon_diagonal_known_answer(ref, cuda, monkeypatch):
    import morph_b200
    import streamtrain.optimizer
    monkeypatch.setattr(streamtrain.optimizer, "HybridMuonAdamW", morph_b200.HybridMuonAdamW)
    model = torch.nn.Sequential(torch.nn.Linear(2, 2, bias=False), torch.nn.LayerNorm(2)).to(cuda)
    optimizer = streamtrain.optimizer.HybridMuonAdamW(model, lr=.02)
    weight = model[0].weight
    before = weight.detach().clone()
    weight.grad = torch.diag(torch.tensor([1., 2.], device=cuda))
    # first Nesterov update = .0975 * grad; the quintic on the normalised diagonal
    diagonal = torch.tensor([.0975, .195], dtype=torch.float64)
    diagonal = diagonal / (diagonal.norm() + 1e-7)
    for _ in range(5):
        diagonal = 3.4445 * diagonal - 4.775 * diagonal ** 3 + 2.0315 * diagonal ** 5
    optimizer.step()
    expected = before * (1 - .02 * .01) - .02 * torch.diag(diagonal.float()).to(cuda)
    delta, want = (weight.detach() - before).double(), (expected - before).double()
    assert float((delta - want).norm() / want.norm()) < 1e-2


# ------------------------------------------------ tests/test_fp16.py:41-72 --

def _fp16_config():
    from morph import MorphConfig
    return MorphConfig(vocab_size=256, d_model=16, num_layers=2, d_ff=32, d_state=4, head_dim=8, d_graph=8,
                       graph_nodes=2, graph_enabled=True)


def _overflow_run(tmp_path, tag):
    """test_fp16.py:59-72: the first reverse pass reports an overflow; DiskDLS
    must halve the scale and retry before anything is written."""
    from morph import MorphModel
    from streamtrain.disk import DiskDLS, DiskState
    torch.manual_seed(21)
    source = MorphModel(_fp16_config())
    tokens = torch.randint(256, (1, 9))
    store = DiskState.create(tmp_path / tag, source, source=source)
    executor = DiskDLS(source, store, "cuda", torch.float16, .001, True)
    original, calls = executor.reverse, []

    def reverse(*args, **kwargs):
        calls.append(executor.loss_scale)
        if len(calls) == 1:
            assert not store.manifest["dirty"] and store.manifest["step"] == 0
            return float("inf"), 5.
        return original(*args, **kwargs)

    executor.reverse = reverse
    t0 = time.perf_counter()
    result = executor.step([tokens])
    return store, executor, calls, result, time.perf_counter() - t0


def test_diskdls_fp16_overflow_retry_on_device_scale(ref, cuda, tmp_path):
    import morph_b200
    base_store, _, base_calls, base_result, _ = _overflow_run(tmp_path, "reference")
    with _Patched():
        store, executor, calls, result, _ = _overflow_run(tmp_path, "patched")
        assert isinstance(executor.scaler, morph_b200.DynamicLossScale)
        # one attribute read is one device round trip; DiskDLS.step reads it once per attempt
        t0 = time.perf_counter()
        for _ in range(100):
            executor.scaler.scale
        per_read_us = (time.perf_counter() - t0) / 100 * 1e6
    assert calls[:2] == [128., 64.] and base_calls[:2] == [128., 64.]
    assert store.manifest["loss_scaler"]["scale"] == 64. == base_store.manifest["loss_scaler"]["scale"]
    assert store.manifest["loss_scaler"] == base_store.manifest["loss_scaler"]
    # test_fp16.py:40's tolerance between two FP16 reverse passes
    assert abs(result["grad_norm"] - base_result["grad_norm"]) < max(1e-4, base_result["grad_norm"] * .01)
    for name in base_store.entries:
        a, b = _entry_planes(base_store, name), _entry_planes(store, name)
        np.testing.assert_allclose(b, a, atol=2e-7, rtol=2e-5, err_msg=name)  # test_fp16.py:49's tolerance
    print(f"DynamicLossScale.scale read: {per_read_us:.1f} us")
    assert per_read_us < 5000


def test_diskdls_fault_mid_write_then_resume(ref, cuda, tmp_path):
    """test_fp16.py:41-50 under the patches: a fault after the first state chunk
    is written, reopen, resume_step: the files equal those of a clean step and
    the persisted loss scaler too."""
    from morph import MorphModel
    from streamtrain.disk import DiskDLS, DiskState
    torch.manual_seed(12)
    source = MorphModel(_fp16_config())
    tokens = torch.randint(256, (1, 9))
    with _Patched():
        store = DiskState.create(tmp_path / "base", source, source=source)
        DiskDLS(source, store, "cuda", torch.float16, .001, True).step([tokens])
        faulty = DiskState.create(tmp_path / "fault", source, source=source)
        executor = DiskDLS(source, faulty, "cuda", torch.float16, .001, True)

        def fail(point):
            if point == "partial_state_write":
                raise RuntimeError("interruption")
        faulty.fault = fail
        with pytest.raises(RuntimeError, match="interruption"):
            executor.step([tokens])
        reopened = DiskState.open(tmp_path / "fault", source)
        DiskDLS(source, reopened, "cuda", torch.float16, .001, True).resume_step()
    for entry in store.entries.values():
        a = np.fromfile(store.root / entry["file"], dtype=np.float32)
        b = np.fromfile(reopened.root / entry["file"], dtype=np.float32)
        np.testing.assert_allclose(a, b, atol=2e-7, rtol=2e-5)
    assert reopened.manifest["loss_scaler"] == store.manifest["loss_scaler"]


# ----------------------------------------- tests/test_sparse_disk.py:16-58 --

def _delta_config():
    from morph.delta_config import DeltaConfig
    return DeltaConfig(vocab_size=256, d_model=8, num_layers=1, d_ff=16, expand=2, d_state=2, head_dim=4,
                       expert_count=3, expert_depth=1, expert_ffn=16, latent_dim=4, graph_enabled=False,
                       proof_enabled=False)


def test_sparse_disk_dls_matches_conditional_adamw(ref, cuda, tmp_path):
    from morph.model.delta import DeltaModel
    from streamtrain.disk import DiskState
    from streamtrain.sparse_disk import SparseDiskDLS
    torch.manual_seed(11)
    cfg = _delta_config()
    original = DeltaModel(cfg)
    reference = copy.deepcopy(original)
    with torch.device("meta"):
        template = DeltaModel(cfg)
    opt = torch.optim.AdamW(reference.parameters(), lr=.002, weight_decay=.01, foreach=False)
    batches = [torch.tensor([[1, 2, 3, 4]]), torch.tensor([[3, 4, 5, 6]])]
    with _Patched():
        store = DiskState.create(tmp_path / "state", template, source=original)
        trainer = SparseDiskDLS(template, store, lr=.002)
        for _ in range(2):
            opt.zero_grad(set_to_none=True)
            for b in batches:
                (reference.loss(b) / len(batches)).backward()
            norm = torch.nn.utils.clip_grad_norm_(reference.parameters(), 1.).item()
            opt.step()
            result = trainer.step(batches)
            assert "_mb_gpu_updater" in store.__dict__  # the updates ran through the GPU updater
            assert result["grad_norm"] == pytest.approx(norm, rel=2e-5, abs=2e-6)
            for name, p in reference.named_parameters():
                torch.testing.assert_close(store.weight(name), p, atol=2e-6, rtol=5e-4, msg=name)
            for name, p in reference.named_parameters():
                expected = int(opt.state[p]["step"]) if p in opt.state else 0
                assert store.manifest.get("parameter_steps", {}).get(name, 0) == expected
        trainer.close()


def test_sparse_disk_dls_fault_and_resume_byte_identical(ref, cuda, tmp_path):
    from morph.model.delta import DeltaModel
    from streamtrain.disk import DiskState
    from streamtrain.sparse_disk import SparseDiskDLS
    torch.manual_seed(13)
    cfg = _delta_config()
    original = DeltaModel(cfg)
    with torch.device("meta"):
        template = DeltaModel(cfg)
    batches = [torch.tensor([[1, 2, 3, 4]])]
    with _Patched():
        a = DiskState.create(tmp_path / "a", template, source=original)
        b = DiskState.create(tmp_path / "b", template, source=original)
        SparseDiskDLS(template, b).step(batches)

        def fault(point):
            if point == "partial_state_write":
                raise OSError("crash")
        a.fault = fault
        with pytest.raises(OSError, match="crash"):
            SparseDiskDLS(template, a).step(batches)
        a = DiskState.open(a.root, template)
        SparseDiskDLS(template, a).resume_step()
    assert a.manifest["parameter_steps"] == b.manifest["parameter_steps"]
    for n in b.entries:
        assert (a.root / a.entries[n]["file"]).read_bytes() == (b.root / b.entries[n]["file"]).read_bytes()


# ------------------------------------------- tests/test_state_cache.py:34-46 --

class _Config:
    def to_dict(self):
        return {"name": "tiny"}


class _Tiny(torch.nn.Module):
    def __init__(self, values):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.tensor(values, dtype=torch.float32))
        self.config = _Config()


def _cache_scenario(tmp_path, tag):
    from streamtrain.disk import DiskState
    from streamtrain.state_cache import CachedDiskState
    values = (1.0, -2.0, 0.5)
    model_a, model_b = _Tiny(values), _Tiny(values)
    plain = DiskState.create(tmp_path / tag / "plain", model_a, source=model_a)
    cached = CachedDiskState.create(tmp_path / tag / "cached", model_b, source=model_b, cache_bytes=36)

    def update_one(store, grad, step, clip):
        store.begin_step()
        store.update("weight", torch.tensor(grad, dtype=torch.float32), step, 0.003, clip, chunk_elements=2)
        store.finish_step()

    for step, grad, clip in [(1, [2.0, -1.0, 0.5], 0.25), (2, None, 1.0), (3, [-0.3, 1.2, 5.0], 0.1)]:
        if grad is not None:
            update_one(plain, grad, step, clip)
            update_one(cached, grad, step, clip)
        else:
            assert torch.equal(plain.weight("weight"), cached.weight("weight"))
    return plain, cached


def test_cached_store_hits_on_device_match_plain_store(ref, cuda, tmp_path):
    base_plain, base_cached = _cache_scenario(tmp_path, "reference")
    with _Patched(cached=True, loss_scale=False):
        plain, cached = _cache_scenario(tmp_path, "patched")
        assert "_mb_gpu_updater" in plain.__dict__ and "_mb_gpu_updater" in cached.__dict__
    assert cached.cache_stats["hits"] >= 1 and cached.cache_stats["cache_bytes"] <= 36
    assert cached.cache_stats["hits"] == base_cached.cache_stats["hits"]
    torch.testing.assert_close(plain.weight("weight"), cached.weight("weight"), rtol=0, atol=0)
    assert (plain.root / plain.entries["weight"]["file"]).read_bytes() == \
        (cached.root / cached.entries["weight"]["file"]).read_bytes()
    # against the unpatched reference (CPU arithmetic): the reference's DiskState-vs-torch tolerance
    np.testing.assert_allclose(_entry_planes(plain, "weight"), _entry_planes(base_plain, "weight"),
                               rtol=5e-4, atol=2e-6)


# ---------------------------------------- morph/training/runner.py:46,100-101 --

def _drop_in_adamw(made):
    import morph_b200

    def factory(params, lr=1e-3, weight_decay=1e-2, foreach=None, **kw):
        opt = morph_b200.AdamW(params, lr=lr, weight_decay=weight_decay, foreach=foreach, **kw)
        made.append(opt)
        return opt
    return factory


def test_resident_runner_with_drop_in_adamw(ref, cuda, tmp_path, monkeypatch):
    from morph import MorphConfig
    from morph.training.runner import train_run
    cfg = MorphConfig(vocab_size=8, d_model=8, num_layers=1, d_ff=16, d_state=2, head_dim=4)
    ids = torch.tensor([[1, 2, 3, 1, 2, 3]])
    kwargs = dict(cfg=cfg, tokens=ids, seed=8, lr=.02, engine="resident", device="cuda", optimizer_name="adamw")
    base = train_run(**kwargs, steps=30)
    made = []
    monkeypatch.setattr(torch.optim, "AdamW", _drop_in_adamw(made))
    uninterrupted = train_run(**kwargs, steps=30)
    assert len(made) == 1 and made[0]._engine is not None  # the runner stepped the drop-in
    # same trajectory as torch's AdamW to within the last bits of each update
    np.testing.assert_allclose(uninterrupted["losses"], base["losses"], rtol=1e-3)
    checkpoint = tmp_path / "resume.pt"
    train_run(**kwargs, steps=12, checkpoint=checkpoint)
    resumed = train_run(**kwargs, steps=30, resume=checkpoint)
    assert uninterrupted["losses"] == resumed["losses"]
    for p, q in zip(uninterrupted["model"].parameters(), resumed["model"].parameters()):
        torch.testing.assert_close(p, q, rtol=0, atol=0)
