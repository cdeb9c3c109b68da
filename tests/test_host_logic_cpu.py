"""Host-side logic that needs no GPU: the bias-correction tables, the disk-rule
step scalars, the Muon batch plan and operand choice, the library's workspace
sizing (host-only C-ABI entry points), the Muon/AdamW partition, the AdamW
constructor's validation and the loss scale's host transitions."""
import math

import numpy as np
import pytest
import torch

from morph_b200 import _lib
from oracle import oracle as orc


def test_bias_correction_tables_match_the_reference_expressions():
    from morph_b200.optim import BiasCorrectionTables
    t = BiasCorrectionTables("cpu")
    t.index(.9, .999, "torch")
    t.index(.9, .95, "torch")
    t.index(.9, .999, "disk")
    tab, n = t.ensure(1)
    assert n == math.ceil(60 * math.log(2) / -math.log(.999)) + 2  # built to saturation up front
    tab = tab.numpy()
    for step in (1, 2, 3, 100, 1023, 5000, 41000):
        assert tab[0, step] == 1 - .9 ** float(step)
        assert tab[1, step] == (1 - .999 ** float(step)) ** 0.5
        assert tab[3, step] == (1 - .95 ** float(step)) ** 0.5
        assert tab[5, step] == math.sqrt(1 - .999 ** float(step))
    assert tab[1, n - 1] == 1.0 and tab[0, n - 1] == 1.0  # saturated: clocks beyond clamp exactly
    again, n2 = t.ensure(10 ** 6)
    assert again is t.tensor and n2 == n  # never rebuilt once saturated


def test_bias_correction_tables_are_bounded_for_beta2_near_one():
    from morph_b200.optim import BiasCorrectionTables
    t = BiasCorrectionTables("cpu")
    t.index(.9, .999999, "torch")
    _, n = t.ensure(1)
    assert n == BiasCorrectionTables.MAX_LENGTH


@pytest.mark.parametrize("lr,step,clip,scale", [(1e-4, 1, 1.0, 1.0), (3e-3, 7, .25, 1024.0), (1e-3, 41000, .5, 3.0)])
def test_disk_host_scalars_match_the_oracle(lr, step, clip, scale):
    from morph_b200.disk import disk_host_scalars
    s = disk_host_scalars(lr, step, clip, scale)
    o = orc.disk_scalars(lr, step)
    for ours, theirs in (("cwd", "cwd"), ("omb1", "omb1"), ("beta2", "b2"), ("omb2", "omb2"), ("bc2s", "bc2s"),
                         ("eps", "eps"), ("nss", "nss")):
        assert getattr(s, ours) == getattr(o, theirs), ours
    assert s.scale == np.float32(scale) and s.coef == np.float32(clip)


def test_muon_batch_plan_and_operands():
    from morph_b200.muon import batch_plan, ns_operand_dtype
    per = _lib.lib().mb_muon_batch_workspace_bytes(1, 4096, 11008)
    assert per > 0 and _lib.lib().mb_muon_batch_workspace_bytes(2, 4096, 11008) > per
    for count in (1, 7, 96, 128, 200):
        for limit in (1, per * 5, 4 << 30):
            sizes = batch_plan(count, 4096, 11008, limit)
            assert sum(sizes) == count
            assert max(sizes) <= max(1, min(_lib.MB_MUON_MAX_BATCH, limit // per))
            assert all(x == sizes[0] for x in sizes[:-1]) and sizes[-1] <= sizes[0]  # evenly filled
    assert batch_plan(0, 64, 64, 1 << 30) == []
    with pytest.raises(ValueError):
        batch_plan(3, 0, 64, 1 << 30)
    assert ns_operand_dtype(48, 80) == _lib.MB_F16 and ns_operand_dtype(4096, 4096, "bf16") == _lib.MB_BF16
    with pytest.raises(ValueError):
        ns_operand_dtype(64, 64, "fp8")


def test_workspace_sizes_are_aligned_and_grow():
    L = _lib.lib()
    sizes = [L.mb_workspace_bytes(n) for n in (1, 2, 100, 8192)]
    assert all(s % 256 == 0 for s in sizes) and sizes == sorted(sizes)
    assert L.mb_accumulate_workspace_bytes() >= 8 * 1024
    assert L.mb_muon_workspace_bytes(0, 64) == 0 and L.mb_muon_workspace_bytes(64, 64) > 0


def test_dtype_codes_and_status_mapping():
    assert _lib.dtype_code(torch.bfloat16) == _lib.MB_BF16 and _lib.dtype_code(None) == _lib.MB_NONE
    with pytest.raises(ValueError):
        _lib.dtype_code(torch.int8)
    with pytest.raises(TimeoutError):
        _lib.check(_lib.MB_ERR_TIMEOUT)


def test_partition_follows_the_reference_rule():
    """streamtrain/optimizer.py:25-31: the weight of every nn.Linear whose
    module name is not exactly 'lm_head' goes to Muon; biases, embeddings,
    norms, the top-level lm_head and anything else go to AdamW, both lists in
    model.parameters() order (tied parameters once)."""
    from morph_b200.muon import partition

    class Block(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.up = torch.nn.Linear(4, 8)
            self.down = torch.nn.Linear(8, 4, bias=False)
            self.norm = torch.nn.LayerNorm(4)
            self.lm_head = torch.nn.Linear(4, 4, bias=False)  # nested: its name is 'blocks.0.lm_head'

    class Model(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.embed = torch.nn.Embedding(10, 4)
            self.blocks = torch.nn.ModuleList([Block(), Block()])
            self.lm_head = torch.nn.Linear(4, 10, bias=False)
            self.lm_head.weight = self.embed.weight  # tied

    model = Model()
    muon, adam = partition(model)
    want_muon = [b.up.weight for b in model.blocks] + [b.down.weight for b in model.blocks] + \
                [b.lm_head.weight for b in model.blocks]
    assert {id(p) for p in muon} == {id(p) for p in want_muon} and len(muon) == len(want_muon)
    order = [id(p) for p in model.parameters()]
    assert [id(p) for p in muon] == sorted((id(p) for p in muon), key=order.index)
    assert [id(p) for p in adam] == [i for i in order if i not in {id(p) for p in muon}]
    assert id(model.embed.weight) in {id(p) for p in adam}


def test_adamw_constructor_rejects_what_torch_rejects():
    """morph_b200.AdamW raises where torch.optim.AdamW does (lr, eps, betas) and
    refuses the torch options the kernels do not implement."""
    from morph_b200 import AdamW
    ps = [torch.nn.Parameter(torch.zeros(4))]
    for kw in (dict(lr=-1e-3), dict(eps=-1.0), dict(betas=(1.0, .999)), dict(betas=(.9, -0.1))):
        with pytest.raises(ValueError):
            torch.optim.AdamW(ps, **kw)
        with pytest.raises(ValueError):
            AdamW(ps, **kw)
    for kw in (dict(amsgrad=True), dict(maximize=True), dict(differentiable=True)):
        with pytest.raises(NotImplementedError):
            AdamW(ps, **kw)
    with pytest.raises(ValueError):
        AdamW(ps, clip_mode="other")
    opt = AdamW(ps, lr=3e-4, betas=(.9, .95), weight_decay=.1)
    ref = torch.optim.AdamW(ps, lr=3e-4, betas=(.9, .95), weight_decay=.1, foreach=False)
    assert set(opt.param_groups[0]) >= {"lr", "betas", "eps", "weight_decay", "amsgrad", "maximize", "foreach",
                                       "capturable", "differentiable", "fused"}
    for k in ("lr", "betas", "eps", "weight_decay", "amsgrad", "maximize"):
        assert opt.param_groups[0][k] == ref.param_groups[0][k], k


def test_loss_scale_host_transitions_follow_the_reference():
    """morph_b200.DynamicLossScale's host-driven overflow()/success() and
    state_dict round trip, on a host-resident record, step for step against the
    restatement of streamtrain/precision.py:6-17 (pinned to the reference's
    golden sequences in test_oracle_cpu.py)."""
    from morph_b200 import DynamicLossScale
    assert DynamicLossScale(device="cpu").scale == 128.0  # precision.py:7 default
    for scale, interval in ((128., 2000), (4., 3), (32768., 2), (1., 1)):
        ours, ref = DynamicLossScale(scale, interval, device="cpu"), orc.DynamicLossScale(scale, interval)
        rng = np.random.default_rng(int(scale) + interval)
        for _ in range(40):
            if rng.random() < .3:
                raised = []
                for s in (ours, ref):
                    try:
                        s.overflow()
                        raised.append(False)
                    except FloatingPointError:
                        raised.append(True)
                assert raised[0] == raised[1]
            else:
                ours.success()
                ref.success()
            assert ours.state_dict() == ref.state_dict()
        other = DynamicLossScale(device="cpu")
        other.load_state_dict(ours.state_dict())
        assert other.state_dict() == ours.state_dict()
