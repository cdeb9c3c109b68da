"""Edge cases of the drop-in AdamW on the GPU, each against the CPU oracle
(torch AdamW arithmetic): parameters without a gradient keep their state and
clock (torch skips them), empty parameters, several parameter groups, clocks
far past the bias-correction tables' saturation, and a checkpoint loaded
mid-training continuing bit for bit. Tolerance as everywhere for AdamW: m and
v bit-exact, w within 1e-6 relative (torch's CPU sqrt may differ by an ulp)."""
import io

import numpy as np
import pytest
import torch

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _close_w(got, want, lr):
    np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-6 * lr)


def _params(cuda, shapes, seed):
    r = orc.rng(seed)
    ps = [torch.nn.Parameter(torch.from_numpy(r.standard_normal(s).astype(np.float32) * np.float32(.02)).to(cuda))
          for s in shapes]
    for p in ps:
        p.grad_dtype = None
    return ps


def test_params_without_grad_keep_state_and_clock(cuda):
    from morph_b200 import AdamW
    shapes = [(300,), (64, 33), (5000,)]
    ps = _params(cuda, shapes, 1)
    opt = AdamW(ps, lr=1e-3, betas=(.9, .95), eps=1e-8, weight_decay=.1)
    ref = [dict(w=p.detach().cpu().numpy().copy(), m=np.zeros(p.shape, np.float32),
                v=np.zeros(p.shape, np.float32), t=0) for p in ps]
    r = orc.rng(2)
    plan = [(0, 1, 2), (0, 2), (1,), (0, 1, 2)]  # which parameters get a gradient each step
    for active in plan:
        for i, p in enumerate(ps):
            if i in active:
                g = r.standard_normal(p.shape).astype(np.float32) * np.float32(1e-3)
                p.grad = torch.from_numpy(g).to(cuda).to(torch.bfloat16)
                rf = ref[i]
                rf["t"] += 1
                orc.adamw_(rf["w"], rf["m"], rf["v"], p.grad.float().cpu().numpy(),
                           orc.adamw_scalars(1e-3, .9, .95, 1e-8, .1, rf["t"]))
            else:
                p.grad = None
        opt.step()
        for i, p in enumerate(ps):
            rf = ref[i]
            _close_w(p.detach().cpu().numpy(), rf["w"], 1e-3)
            if rf["t"]:
                np.testing.assert_array_equal(opt.state[p]["exp_avg"].cpu().numpy(), rf["m"])
                np.testing.assert_array_equal(opt.state[p]["exp_avg_sq"].cpu().numpy(), rf["v"])
                assert int(float(opt.state[p]["step"])) == rf["t"]


def test_empty_parameter_alongside_others(cuda):
    from morph_b200 import AdamW
    ps = _params(cuda, [(0,), (17,), (0, 8), (4096,)], 3)
    opt = AdamW(ps, lr=1e-3, weight_decay=.01, low_precision=torch.bfloat16)
    r = orc.rng(4)
    ws = [p.detach().cpu().numpy().copy() for p in ps]
    ms = [np.zeros_like(w) for w in ws]
    vs = [np.zeros_like(w) for w in ws]
    for step in (1, 2):
        for p in ps:
            p.grad = torch.from_numpy(r.standard_normal(p.shape).astype(np.float32) * np.float32(1e-3)).to(cuda)
        opt.step()
        for i, p in enumerate(ps):
            orc.adamw_(ws[i], ms[i], vs[i], p.grad.cpu().numpy(), orc.adamw_scalars(1e-3, .9, .999, 1e-8, .01, step))
            _close_w(p.detach().cpu().numpy(), ws[i], 1e-3)
            assert int(float(opt.state[p]["step"])) == step
            assert opt.low_precision_copies[p].shape == p.shape


def test_several_param_groups(cuda):
    from morph_b200 import AdamW
    ps = _params(cuda, [(1000,), (3000,), (77,), (2048,)], 5)
    hyper = [dict(lr=1e-3, betas=(.9, .95), weight_decay=.1), dict(lr=3e-4, betas=(.8, .999), weight_decay=0.0)]
    opt = AdamW([dict(params=ps[:2], **hyper[0]), dict(params=ps[2:], **hyper[1])], eps=1e-8)
    r = orc.rng(6)
    ws = [p.detach().cpu().numpy().copy() for p in ps]
    ms = [np.zeros_like(w) for w in ws]
    vs = [np.zeros_like(w) for w in ws]
    for step in (1, 2, 3):
        for p in ps:
            p.grad = torch.from_numpy(r.standard_normal(p.shape).astype(np.float32) * np.float32(1e-3)).to(cuda)
        opt.step()
        for i, p in enumerate(ps):
            h = hyper[0 if i < 2 else 1]
            orc.adamw_(ws[i], ms[i], vs[i], p.grad.cpu().numpy(),
                       orc.adamw_scalars(h["lr"], h["betas"][0], h["betas"][1], 1e-8, h["weight_decay"], step))
            _close_w(p.detach().cpu().numpy(), ws[i], h["lr"])
            np.testing.assert_array_equal(opt.state[p]["exp_avg"].cpu().numpy(), ms[i])


@pytest.mark.parametrize("start", [1023, 5000, 50000, 10 ** 6])
def test_clocks_past_table_growth_and_saturation(cuda, start):
    """A checkpoint at clock `start` (past the first table, past beta2's
    saturation): the next steps use bias corrections of start+1, start+2."""
    from morph_b200 import AdamW
    ps = _params(cuda, [(5000,)], 7)
    p = ps[0]
    r = orc.rng(8)
    m0 = r.standard_normal(p.shape).astype(np.float32) * np.float32(1e-3)
    v0 = np.abs(r.standard_normal(p.shape).astype(np.float32)) * np.float32(1e-6)
    opt = AdamW(ps, lr=1e-3, betas=(.9, .999), weight_decay=.01)
    sd = dict(state={0: dict(step=torch.tensor(float(start)), exp_avg=torch.from_numpy(m0),
                             exp_avg_sq=torch.from_numpy(v0))},
              param_groups=[dict(opt.state_dict()["param_groups"][0])])
    opt.load_state_dict(sd)
    w, m, v = p.detach().cpu().numpy().copy(), m0.copy(), v0.copy()
    for t in (start + 1, start + 2):
        g = r.standard_normal(p.shape).astype(np.float32) * np.float32(1e-3)
        p.grad = torch.from_numpy(g).to(cuda)
        opt.step()
        orc.adamw_(w, m, v, g, orc.adamw_scalars(1e-3, .9, .999, 1e-8, .01, t))
        _close_w(p.detach().cpu().numpy(), w, 1e-3)
        np.testing.assert_array_equal(opt.state[p]["exp_avg_sq"].cpu().numpy(), v)
        assert int(float(opt.state[p]["step"])) == t


def test_checkpoint_mid_training_continues_bit_for_bit(cuda):
    from morph_b200 import AdamW
    shapes = [(300, 7), (4099,)]
    a = _params(cuda, shapes, 9)
    b = _params(cuda, shapes, 9)
    oa = AdamW(a, lr=1e-3, weight_decay=.05, max_norm=1.0)
    r = orc.rng(10)
    grads = [[torch.from_numpy(r.standard_normal(s).astype(np.float32) * np.float32(.3)).to(cuda) for s in shapes]
             for _ in range(5)]
    for gs in grads[:3]:
        for p, g in zip(a, gs):
            p.grad = g
        oa.step()
    buf = io.BytesIO()  # a checkpoint file: the loaded state does not alias the live one
    torch.save(oa.state_dict(), buf)
    buf.seek(0)
    sd = torch.load(buf, weights_only=True)
    for pb, pa in zip(b, a):
        pb.data.copy_(pa.data)
    ob = AdamW(b, lr=1e-3, weight_decay=.05, max_norm=1.0)
    ob.load_state_dict(sd)
    for gs in grads[3:]:
        for opt, ps in ((oa, a), (ob, b)):
            for p, g in zip(ps, gs):
                p.grad = g.clone()
            opt.step()
    for pa, pb in zip(a, b):
        assert torch.equal(pa, pb)
        assert torch.equal(oa.state[pa]["exp_avg_sq"], ob.state[pb]["exp_avg_sq"])
        assert int(float(oa.state[pa]["step"])) == int(float(ob.state[pb]["step"])) == 5


def test_step_captured_in_a_cuda_graph_replays_like_eager_steps(cuda):
    """AdamW.step (sync=False) launches kernels only: captured once in a CUDA
    graph it replays as many steps as wanted (device clocks, clip and copies
    advance on the device), bit-identical to eager steps."""
    from morph_b200 import AdamW
    shapes = [(300, 7), (4099,), (64, 64)]
    a = _params(cuda, shapes, 21)
    b = _params(cuda, shapes, 21)
    kw = dict(lr=1e-3, betas=(.9, .95), weight_decay=.1, max_norm=1.0, low_precision=torch.bfloat16)
    oa, ob = AdamW(a, **kw), AdamW(b, **kw)
    grads = [torch.zeros(s, device=cuda, dtype=torch.bfloat16) for s in shapes]  # static grad buffers
    for p, g in zip(a, grads):
        p.grad = g
    gen = torch.Generator(device=cuda).manual_seed(22)

    def fresh():
        return [(torch.randn(s, device=cuda, generator=gen) * .3).to(torch.bfloat16) for s in shapes]

    def eager_b(gs):
        for p, g in zip(b, gs):
            p.grad = g.clone()
        ob.step()

    gs = fresh()  # step 1 eager on both (builds the state and the launch plan)
    for buf, g in zip(grads, gs):
        buf.copy_(g)
    oa.step()
    eager_b(gs)
    side = torch.cuda.Stream(cuda)
    side.wait_stream(torch.cuda.current_stream(cuda))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side), torch.cuda.graph(graph, stream=side):
        oa.step()
    torch.cuda.current_stream(cuda).wait_stream(side)
    for _ in range(4):
        gs = fresh()
        for buf, g in zip(grads, gs):
            buf.copy_(g)
        graph.replay()
        eager_b(gs)
    torch.cuda.synchronize(cuda)
    for pa, pb in zip(a, b):
        assert torch.equal(pa, pb)
        assert torch.equal(oa.state[pa]["exp_avg_sq"], ob.state[pb]["exp_avg_sq"])
        assert torch.equal(oa.low_precision_copies[pa], ob.low_precision_copies[pb])
        assert int(float(oa.state[pa]["step"])) == int(float(ob.state[pb]["step"])) == 5
    assert oa.last_step()["clip_coef"] == ob.last_step()["clip_coef"] < 1.0


def test_thousands_of_ragged_tensors_against_oracle(cuda):
    """3000 tensors of random sizes (0 .. 5000, some views off the 16-byte grid):
    many segment changes per CTA, bulk-staged and direct tiles mixed, BF16
    grads and copies; bit-exact with the oracle over two steps."""
    from morph_b200 import AdamW
    r = orc.rng(123)
    sizes = [int(x) for x in r.integers(0, 5001, size=3000)]
    base = torch.from_numpy(r.standard_normal(sum(sizes) + 4 * len(sizes)).astype(np.float32)
                            * np.float32(.02)).to(cuda)
    ps, off = [], 0
    for i, n in enumerate(sizes):
        if i % 3 == 0:  # disjoint views of one flat buffer at arbitrary (unaligned) offsets
            o = off + int(r.integers(0, 4))
            ps.append(torch.nn.Parameter(base[o:o + n]))
            off = o + n
        else:
            ps.append(torch.nn.Parameter(torch.from_numpy(r.standard_normal(n).astype(np.float32)
                                                          * np.float32(.02)).to(cuda)))
    for p in ps:
        p.grad_dtype = None
    opt = AdamW(ps, lr=1e-3, betas=(.9, .95), weight_decay=.1, low_precision=torch.bfloat16)
    ws = [p.detach().cpu().numpy().copy() for p in ps]
    ms = [np.zeros_like(w) for w in ws]
    vs = [np.zeros_like(w) for w in ws]
    for step in (1, 2):
        gs = [torch.from_numpy(r.standard_normal(p.numel()).astype(np.float32) * np.float32(1e-3)).bfloat16()
              for p in ps]
        for p, g in zip(ps, gs):
            p.grad = g.to(cuda).view(p.shape)
        opt.step()
        got_w = [p.detach().cpu().numpy() for p in ps]
        got_c = [opt.low_precision_copies[p].float().cpu().numpy() for p in ps]
        for i, g in enumerate(gs):
            orc.adamw_(ws[i], ms[i], vs[i], g.float().numpy(), orc.adamw_scalars(1e-3, .9, .95, 1e-8, .1, step))
            np.testing.assert_array_equal(got_w[i], ws[i])
            np.testing.assert_array_equal(got_c[i], torch.from_numpy(ws[i]).bfloat16().float().numpy())
