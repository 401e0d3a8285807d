"""Variable all-to-all token dispatch (gloo, 2 ranks)."""
import torch

from dist_utils import run_ranks


def _dispatch_worker(rank, world):
    import torch.distributed as dist

    from parallel_b200.parallel.model_parallel import ExpertPartition, TokenDispatcher
    from parallel_b200.profiling import (collective_phase, configure_collective_profiling,
                                         finish_collective_profile_step, start_collective_profile_step)

    configure_collective_profiling(enabled=True)
    start_collective_profile_step()
    part = ExpertPartition(num_experts=4, ep_size=2, ep_rank=rank)
    disp = TokenDispatcher(part, dist.group.WORLD)
    T, K, H = 3, 2, 5
    torch.manual_seed(rank)
    hidden = torch.randn(T, H, requires_grad=True)
    # rank 1 routes nothing to rank 0's experts: rank 0 receives only its own routes
    idx = torch.tensor([[0, 3], [1, 2], [3, 0]]) if rank == 0 else torch.tensor([[2, 3], [3, 2], [2, 3]])
    scores = torch.rand(T, K)
    with collective_phase("forward"):
        h, e, s, state = disp.dispatch(hidden, idx, scores)
        assert int(e.max()) < part.local_count
        out = disp.combine(h, state)
    torch.testing.assert_close(out, hidden * K)  # identity experts: each token returns K times
    out.sum().backward()
    torch.testing.assert_close(hidden.grad, torch.full_like(hidden, float(K)))
    lines = finish_collective_profile_step()
    assert any("op=ep_all_to_all" in l and "mode=dispatch_hidden" in l for l in lines)


def test_dispatch_combine_identity_and_grads():
    run_ranks(_dispatch_worker, 2)


def _empty_receiver_worker(rank, world):
    import torch.distributed as dist

    from parallel_b200.parallel.model_parallel import ExpertPartition, TokenDispatcher

    part = ExpertPartition(num_experts=4, ep_size=2, ep_rank=rank)
    disp = TokenDispatcher(part, dist.group.WORLD)
    T, K, H = 4, 2, 3
    torch.manual_seed(10 + rank)
    hidden = torch.randn(T, H, requires_grad=True)
    idx = torch.tensor([[2, 3]] * T)  # every route of both ranks goes to rank 1's experts
    scores = torch.rand(T, K)
    h, e, s, state = disp.dispatch(hidden, idx, scores)
    if rank == 0:
        assert h.shape[0] == 0 and e.numel() == 0  # rank 0 receives nothing
    else:
        assert h.shape[0] == 2 * T * K
    out = disp.combine(h * 2, state)
    torch.testing.assert_close(out, hidden * 2 * K)
    out.sum().backward()
    torch.testing.assert_close(hidden.grad, torch.full_like(hidden, 2.0 * K))


def test_dispatch_with_a_rank_receiving_no_tokens():
    run_ranks(_empty_receiver_worker, 2)
