"""Device-resident MoE routing (csrc/moe.cu + the grouped GEMM's device tile
count) against fp32 PyTorch restatements, on one GPU."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel_err(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def _no_device_error():
    from parallel_b200.ops._ext import check_device_errors

    torch.cuda.synchronize()
    check_device_errors()


def _expected_plan(topi, mat, my_row, E_loc, ep_rank, local_only):
    """The padded expert-major layout and each route's (owner, row), computed
    with plain Python from the histogram matrix."""
    E = mat.shape[1]
    owners = E // E_loc
    m = mat.long().tolist()
    base, own = {}, None
    for d in range(owners):
        off, cnts, offs = 0, [], []
        for j in range(E_loc):
            e = d * E_loc + j
            total = sum(m[s][e] for s in range(len(m)))
            base[e] = off + sum(m[s][e] for s in range(my_row))
            cnts.append(total)
            offs.append(off)
            off += 128 * -(-max(total, 1) // 128)
        if d == ep_rank:
            own = (cnts, offs, off // 128)
    seen = {}
    route_owner, route_row = [], []
    for e in topi.reshape(-1).tolist():
        d = e // E_loc
        if local_only and d != ep_rank:
            route_owner.append(-1)
            route_row.append(-1)
            continue
        route_owner.append(0 if local_only else d)
        route_row.append(base[e] + seen.get(e, 0))
        seen[e] = seen.get(e, 0) + 1
    return route_owner, route_row, own


@pytest.mark.parametrize("local_only", [False, True])
def test_route_plan_matches_python(local_only):
    from parallel_b200.ops._ext import ext
    from parallel_b200.ops.moe import plan_routes, tiles_capacity

    torch.manual_seed(3)
    T, K, E, W, me = 1000, 8, 128, 4, 2
    E_loc = E // W
    topi = torch.stack([torch.randperm(E)[:K] for _ in range(T)]).cuda()
    if local_only:
        mat = torch.empty(1, E, device="cuda")
        ext().moe_hist(topi, mat, 0)
        row, routes_in = 0, T * K
    else:
        mat = torch.empty(W, E, device="cuda")
        ext().moe_hist(topi, mat, me)
        assert mat[me].sum().item() == T * K and mat[0].abs().sum().item() == 0
        # the other ranks' histograms, as the all-reduce would deliver them
        for s in range(W):
            if s != me:
                mat[s] = torch.bincount(torch.randint(0, E, (T * K,)), minlength=E).float().cuda()
        row, routes_in = me, W * T * K
    cap = tiles_capacity(routes_in, E_loc)
    plan = plan_routes(topi, mat, row, E_loc, me, local_only, cap)
    _no_device_error()
    owner, rrow, (cnts, offs, tiles) = _expected_plan(topi.cpu(), mat.cpu(), row, E_loc, me, local_only)
    assert plan.route_owner.tolist() == owner
    assert plan.route_row.tolist() == rrow
    assert plan.own_cnt.tolist() == cnts and plan.own_off.tolist() == offs
    assert int(plan.n_tiles.item()) == tiles
    te = plan.tile_expert[:tiles].tolist()
    assert te == [j for j in range(E_loc) for _ in range(-(-max(cnts[j], 1) // 128))]
    kr = plan.krange.tolist()
    assert kr == [[o, o + 64 * -(-max(c, 1) // 64)] for o, c in zip(offs, cnts)]


def _fp32_experts(x, w, idx, w_gu, w_d):
    out = torch.zeros_like(x)
    for e in range(w_gu.shape[0]):
        tok, kk = torch.where(idx == e)
        if tok.numel() == 0:
            continue
        g, u = (x[tok] @ w_gu[e].t()).chunk(2, dim=-1)
        y = (torch.nn.functional.silu(g) * u) @ w_d[e].t()
        out = out.index_add(0, tok, y * w[tok, kk, None])
    return out


@pytest.mark.parametrize("T,E,K,I,skew", [(300, 16, 4, 128, 0.0), (1000, 64, 8, 384, 3.0), (129, 8, 2, 256, 6.0)])
def test_routed_experts_match_fp32(T, E, K, I, skew):
    """Forward and all gradients of dispatch -> expert MLPs -> weighted combine
    against fp32 PyTorch; the skewed router leaves experts without routes."""
    from parallel_b200.ops.moe import LocalExpertTransport, routed_experts

    torch.manual_seed(11)
    H = 256
    logits = torch.randn(T, E) + torch.randn(E) * skew
    w, idx = torch.softmax(logits, -1).topk(K, -1)
    x = (torch.randn(T, H) * 0.5).cuda().to(torch.bfloat16).requires_grad_(True)
    wts = w.cuda().requires_grad_(True)
    w_gu = (torch.randn(E, 2 * I, H) / math.sqrt(H)).cuda().to(torch.bfloat16).requires_grad_(True)
    w_d = (torch.randn(E, H, I) / math.sqrt(I)).cuda().to(torch.bfloat16).requires_grad_(True)
    out = routed_experts(x, wts, idx.cuda(), w_gu, w_d, LocalExpertTransport(E))
    g = torch.randn(T, H).cuda().to(torch.bfloat16)
    out.backward(g)
    _no_device_error()
    xf, wf = x.detach().float().requires_grad_(True), wts.detach().clone().requires_grad_(True)
    guf, df = w_gu.detach().float().requires_grad_(True), w_d.detach().float().requires_grad_(True)
    ref = _fp32_experts(xf, wf, idx.cuda(), guf, df)
    ref.backward(g.float())
    assert _rel_err(out, ref) < 2e-2
    assert _rel_err(x.grad, xf.grad) < 3e-2
    assert _rel_err(wts.grad, wf.grad) < 3e-2
    assert _rel_err(w_gu.grad, guf.grad) < 3e-2
    assert _rel_err(w_d.grad, df.grad) < 3e-2
    unused = sorted(set(range(E)) - set(idx.reshape(-1).tolist()))
    for e in unused:  # experts without routes get exactly zero weight gradients
        assert w_gu.grad[e].abs().max().item() == 0 and w_d.grad[e].abs().max().item() == 0
    if skew >= 3.0:
        assert unused, "the skewed case should leave some expert without routes"


def test_replicated_token_layout_keeps_only_local_experts():
    """local_only: routes to other ranks' experts are dropped (zero output and
    zero weight gradient), the rest equals the full computation restricted to
    this rank's experts."""
    from parallel_b200.ops.moe import LocalExpertTransport, routed_experts

    torch.manual_seed(5)
    T, E, K, H, I, W, me = 200, 16, 4, 128, 128, 4, 1
    E_loc = E // W
    w, idx = torch.softmax(torch.randn(T, E), -1).topk(K, -1)
    x = torch.randn(T, H).cuda().to(torch.bfloat16).requires_grad_(True)
    wts = w.cuda().requires_grad_(True)
    w_gu = (torch.randn(E_loc, 2 * I, H) / math.sqrt(H)).cuda().to(torch.bfloat16).requires_grad_(True)
    w_d = (torch.randn(E_loc, H, I) / math.sqrt(I)).cuda().to(torch.bfloat16).requires_grad_(True)
    tr = LocalExpertTransport(E_loc, num_experts=E, ep_rank=me, local_only=True)
    out = routed_experts(x, wts, idx.cuda(), w_gu, w_d, tr)
    out.float().square().sum().backward()
    _no_device_error()
    local = (idx // E_loc) == me
    lidx = torch.where(local, idx - me * E_loc, torch.full_like(idx, E_loc)).cuda()
    xf, wf = x.detach().float().requires_grad_(True), wts.detach().clone().requires_grad_(True)
    ref = _fp32_experts(xf, wf * local.cuda(), lidx, w_gu.detach().float(), w_d.detach().float())
    ref.square().sum().backward()
    assert _rel_err(out, ref) < 2e-2
    assert _rel_err(x.grad, xf.grad) < 3e-2
    assert _rel_err(wts.grad, wf.grad) < 3e-2
    assert wts.grad[~local.cuda()].abs().max().item() == 0


def test_routed_experts_replay_in_a_cuda_graph():
    """Captured once, replayed with different routings of the same shape: the
    results follow eager execution, so no routing size reaches the host."""
    from parallel_b200.ops.moe import LocalExpertTransport, routed_experts

    torch.manual_seed(21)
    T, E, K, H, I = 512, 32, 4, 256, 128
    x = torch.randn(T, H).cuda().to(torch.bfloat16)
    w_gu = (torch.randn(E, 2 * I, H) / math.sqrt(H)).cuda().to(torch.bfloat16).requires_grad_(True)
    w_d = (torch.randn(E, H, I) / math.sqrt(I)).cuda().to(torch.bfloat16).requires_grad_(True)
    tr = LocalExpertTransport(E)
    wts = torch.zeros(T, K, device="cuda")
    idx = torch.zeros(T, K, dtype=torch.int64, device="cuda")
    xin = x.clone().requires_grad_(True)

    def routing(seed, skew):
        g = torch.Generator().manual_seed(seed)
        w, i = torch.softmax(torch.randn(T, E, generator=g) + torch.randn(E, generator=g) * skew, -1).topk(K, -1)
        return w.cuda(), i.cuda()

    def step():
        for p in (xin, w_gu, w_d):
            p.grad = None
        out = routed_experts(xin, wts.detach().requires_grad_(True), idx, w_gu, w_d, tr)
        out.float().square().sum().backward()
        return out

    w0, i0 = routing(0, 0.0)
    wts.copy_(w0)
    idx.copy_(i0)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()  # warm-up on the capture stream
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out_g = step()
    torch.cuda.current_stream().wait_stream(s)
    # the graph writes its gradients into the tensors the capture produced
    graph_grads = (xin.grad, w_gu.grad, w_d.grad)
    for seed, skew in [(1, 0.0), (2, 4.0)]:
        w1, i1 = routing(seed, skew)
        wts.copy_(w1)
        idx.copy_(i1)
        graph.replay()
        torch.cuda.synchronize()
        got = (out_g.clone(),) + tuple(t.clone() for t in graph_grads)
        eager = step()
        torch.cuda.synchronize()
        assert _rel_err(got[0], eager) < 1e-3
        assert _rel_err(got[1], xin.grad) < 1e-3
        assert _rel_err(got[2], w_gu.grad) < 1e-3
        assert _rel_err(got[3], w_d.grad) < 1e-3
    _no_device_error()
    del graph
