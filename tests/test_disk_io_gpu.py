"""DiskState.update on a (3, size) state file with the arithmetic on the GPU:
the file after the update is bit-exact with the oracle's disk.py:203-223 on the
same planes, the fault hook runs once per reference chunk after that chunk is
written, and a hook that raises leaves exactly the chunks before it updated."""
import numpy as np
import pytest
import torch

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


class FileStore:
    """The parts of the reference's DiskState the updater uses: root, entries, fault."""

    def __init__(self, root, arrays, fail_at=None):
        self.root = root
        self.entries = {}
        self.calls = 0
        self.fail_at = fail_at
        for name, planes in arrays.items():
            path = root / f"{name}.bin"
            planes.astype(np.float32).tofile(path)
            self.entries[name] = {"file": path.name, "size": planes.shape[1]}

    def fault(self, label):
        assert label == "partial_state_write"
        self.calls += 1
        if self.fail_at is not None and self.calls == self.fail_at:
            raise RuntimeError("injected fault")

    def planes(self, name):
        e = self.entries[name]
        return np.fromfile(self.root / e["file"], dtype=np.float32).reshape(3, e["size"])


def _planes(n, seed):
    r = orc.rng(seed)
    w = r.standard_normal(n).astype(np.float32) * np.float32(.02)
    m = r.standard_normal(n).astype(np.float32) * np.float32(1e-3)
    v = np.abs(r.standard_normal(n).astype(np.float32)) * np.float32(1e-6)
    return np.stack([w, m, v])


def _oracle(planes, g32, step, lr, clip):
    w, m, v = (planes[i].copy() for i in range(3))
    orc.adamw_(w, m, v, orc.grad_prepare(g32, coef=clip), orc.disk_scalars(lr, step))
    return np.stack([w, m, v])


@pytest.mark.parametrize("where,gdt", [("cpu", torch.float32), ("cuda", torch.bfloat16), ("cuda", torch.float16)])
@pytest.mark.parametrize("n,chunk,window", [(10_007, 1000, 4000), (3_000_001, 1 << 20, 1 << 24), (5, 1 << 20, 1 << 24)])
def test_file_update_matches_oracle(cuda, tmp_path, where, gdt, n, chunk, window):
    from morph_b200.disk_io import install
    planes = _planes(n, n)
    store = FileStore(tmp_path, {"layer": planes})
    install(store, cuda, window_elements=window)
    g = torch.from_numpy(orc.rng(n + 1).standard_normal(n).astype(np.float32) * np.float32(1e-3)).to(gdt)
    store.update("layer", g.to(where if where == "cpu" else cuda), 3, 1e-3, .7, chunk_elements=chunk)
    torch.cuda.synchronize()
    ref = _oracle(planes, g.float().numpy(), 3, 1e-3, .7)
    np.testing.assert_array_equal(store.planes("layer"), ref)
    assert store.calls == -(-n // chunk)


def test_fault_mid_update_leaves_the_chunks_before_it(cuda, tmp_path):
    from morph_b200.disk_io import install
    n, chunk = 10_007, 1000
    planes = _planes(n, 9)
    store = FileStore(tmp_path, {"layer": planes}, fail_at=5)
    install(store, cuda, window_elements=3000)
    g = torch.from_numpy(orc.rng(10).standard_normal(n).astype(np.float32) * np.float32(1e-3))
    with pytest.raises(RuntimeError, match="injected"):
        store.update("layer", g, 2, 1e-3, 1.0, chunk_elements=chunk)
    torch.cuda.synchronize()
    ref = _oracle(planes, g.numpy(), 2, 1e-3, 1.0)
    got = store.planes("layer")
    np.testing.assert_array_equal(got[:, :5 * chunk], ref[:, :5 * chunk])
    np.testing.assert_array_equal(got[:, 5 * chunk:], planes[:, 5 * chunk:])


def test_two_steps_two_entries(cuda, tmp_path):
    from morph_b200.disk_io import install
    arrays = {"a": _planes(5000, 1), "b": _planes(777, 2)}
    store = FileStore(tmp_path, arrays)
    install(store, cuda, window_elements=2048)
    ref = {k: v.copy() for k, v in arrays.items()}
    for step in (1, 2):
        for name, p in arrays.items():
            g = torch.from_numpy(orc.rng(step * 10 + len(name)).standard_normal(p.shape[1]).astype(np.float32))
            store.update(name, g, step, 1e-4, .5, chunk_elements=1000)
            ref[name] = _oracle(ref[name], g.numpy(), step, 1e-4, .5)
    torch.cuda.synchronize()
    for name in arrays:
        np.testing.assert_array_equal(store.planes(name), ref[name])


def test_patch_class_routes_every_instance(cuda, tmp_path):
    """patch_class swaps a store class's update for the GPU one (one updater per
    instance) and restores it."""
    from morph_b200.disk_io import patch_class

    class Store(FileStore):
        def update(self, *args, **kwargs):
            raise AssertionError("the original update must not run while patched")

    n = 3000
    planes = _planes(n, 41)
    s1 = Store(tmp_path, {"a": planes})
    restore = patch_class(Store, cuda, window_elements=1024)
    try:
        g = torch.from_numpy(orc.rng(42).standard_normal(n).astype(np.float32))
        s1.update("a", g, 1, 1e-3, .5, chunk_elements=1000)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(s1.planes("a"), _oracle(planes, g.numpy(), 1, 1e-3, .5))
        assert s1.calls == 3
    finally:
        restore()
    with pytest.raises(AssertionError):
        s1.update("a", g, 2, 1e-3, .5)


class CachedFileStore(FileStore):
    """The parts of the reference's CachedDiskState the cached patch uses:
    a RAM cache of (3, size) planes, its lock, counters and _drop."""

    def __init__(self, root, arrays, cached, fail_at=None):
        import collections
        import threading
        super().__init__(root, arrays, fail_at)
        self._cache_lock = threading.RLock()
        self._cache = collections.OrderedDict((n, self.planes(n).copy()) for n in cached)
        self._cache_stats = {"hits": 0, "misses": 0, "estimated_bytes_avoided": 0}
        self.dropped = []

    def update(self, *args, **kwargs):
        raise AssertionError("the original update must not run while patched")

    def _drop(self, name):
        self._cache.pop(name, None)
        self.dropped.append(name)


def test_patch_cached_class_hit_and_miss(cuda, tmp_path):
    """state_cache.py:103-140 semantics: a hit updates the RAM copy and the
    file (byte-identical to each other and to the oracle), a miss updates the
    file only; the counters move as the reference's do."""
    from morph_b200.disk_io import patch_cached_class
    arrays = {"hot": _planes(5000, 51), "cold": _planes(7000, 52)}
    store = CachedFileStore(tmp_path, arrays, cached=["hot"])
    restore = patch_cached_class(CachedFileStore, cuda, window_elements=2048)
    try:
        ref = {k: v.copy() for k, v in arrays.items()}
        for step in (1, 2):
            for name, p in arrays.items():
                g = torch.from_numpy(orc.rng(step * 7 + len(name)).standard_normal(p.shape[1]).astype(np.float32))
                store.update(name, g, step, 1e-3, .5, chunk_elements=1000)
                ref[name] = _oracle(ref[name], g.numpy(), step, 1e-3, .5)
        torch.cuda.synchronize()
        for name in arrays:
            np.testing.assert_array_equal(store.planes(name), ref[name])
        np.testing.assert_array_equal(store._cache["hot"], ref["hot"])
        assert store._cache_stats["hits"] == 2 and store._cache_stats["misses"] == 2
    finally:
        restore()


def test_patch_cached_class_fault_drops_the_entry(cuda, tmp_path):
    from morph_b200.disk_io import patch_cached_class
    n, chunk = 5000, 1000
    planes = _planes(n, 53)
    store = CachedFileStore(tmp_path, {"hot": planes}, cached=["hot"], fail_at=3)
    restore = patch_cached_class(CachedFileStore, cuda, window_elements=2000)
    try:
        g = torch.from_numpy(orc.rng(54).standard_normal(n).astype(np.float32))
        with pytest.raises(RuntimeError, match="injected"):
            store.update("hot", g, 1, 1e-3, 1.0, chunk_elements=chunk)
        torch.cuda.synchronize()
        assert store.dropped == ["hot"] and "hot" not in store._cache
        ref = _oracle(planes, g.numpy(), 1, 1e-3, 1.0)
        got = store.planes("hot")
        np.testing.assert_array_equal(got[:, :3 * chunk], ref[:, :3 * chunk])
        np.testing.assert_array_equal(got[:, 3 * chunk:], planes[:, 3 * chunk:])
    finally:
        restore()
