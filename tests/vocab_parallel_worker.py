"""One rank of the two-GPU vocabulary-parallel LM-head check (launched by
tests/test_gpu_vocab_parallel.py::test_two_gpu_vocab_parallel through
torchrun): every rank holds the same hidden states and its half of the
weight rows, runs vocab_parallel_lm_head_loss over NCCL (fused and staged
forms, with rows that take the exact full-row path), and compares the loss,
hidden.grad and its slice of the weight gradient with the one-GPU LM head on
the whole weight."""
import datetime
import os
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [REPO, os.path.join(REPO, "fast-familywise-loss_b200")]

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from fwloss_b200.lm_head import fw_lm_head_loss  # noqa: E402
from fwloss_b200.sharded import even_col_start  # noqa: E402
from fwloss_b200.vocab_parallel import vocab_parallel_lm_head_loss  # noqa: E402


def check(impl, dev, rank, world):
    B, D, C = 300, 256, 20000
    g = torch.Generator(device=dev).manual_seed(11)
    hidden = (torch.randn(B, D, generator=g, device=dev) / D ** 0.5 * 4).to(torch.bfloat16)
    weight = torch.randn(C, D, generator=g, device=dev).to(torch.bfloat16)
    target = torch.randint(0, C, (B,), generator=g, device=dev)
    hidden[7] = 0  # constant logits: exact full-row path
    cs = even_col_start(C, world)
    h = hidden.clone().requires_grad_(True)
    w = weight[cs[rank]:cs[rank + 1]].clone().requires_grad_(True)
    loss = vocab_parallel_lm_head_loss(h, w, target, cs, impl=impl, K=16)
    loss.backward()
    h1 = hidden.clone().requires_grad_(True)
    w1 = weight.clone().requires_grad_(True)
    ref = fw_lm_head_loss(h1, w1, target, impl=impl, K=16)
    ref.backward()
    ok = abs(loss.float().item() - ref.float().item()) <= 1e-2 * max(1.0, abs(ref.float().item()))
    ok &= torch.allclose(h.grad.float(), h1.grad.float(), rtol=2e-2, atol=1e-5)
    ok &= torch.allclose(w.grad.float(), w1.grad[cs[rank]:cs[rank + 1]].float(), rtol=2e-2, atol=1e-5)
    print(f"rank {rank} {impl}: loss {loss.float().item():.6f} ref {ref.float().item():.6f} ok={ok}", flush=True)
    return ok


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    rank, world = dist.get_rank(), dist.get_world_size()
    ok = check("fused", dev, rank, world) & check("staged", dev, rank, world)
    flag = torch.tensor([0 if ok else 1], device=dev)
    dist.all_reduce(flag)
    dist.destroy_process_group()
    sys.exit(int(flag.item() != 0))


if __name__ == "__main__":
    main()
