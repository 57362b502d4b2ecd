"""torch DDP over the commux backend: gradients of a small MLP must equal the
single-process gradient of the concatenated batch (the reference backend
cannot run DDP: no allgather, no Work::getFuture)."""
import torch.nn as nn

from common import Checker, init, torch

rank, world, dev = init()
c = Checker(rank)
torch.manual_seed(0)
model = nn.Sequential(nn.Linear(16, 32), nn.ReLU(), nn.Linear(32, 4)).to(dev)
ref = nn.Sequential(nn.Linear(16, 32), nn.ReLU(), nn.Linear(32, 4)).to(dev)
ref.load_state_dict(model.state_dict())
ddp = nn.parallel.DistributedDataParallel(model, bucket_cap_mb=0.001)
g = torch.Generator().manual_seed(123)
xs = torch.randn(world * 8, 16, generator=g).to(dev)
ys = torch.randn(world * 8, 4, generator=g).to(dev)
loss = ((ddp(xs[rank * 8:(rank + 1) * 8]) - ys[rank * 8:(rank + 1) * 8]) ** 2).mean()
loss.backward()
rloss = ((ref(xs) - ys) ** 2).view(world, 8, 4).mean(dim=(1, 2)).mean()
rloss.backward()
for (n, p), q in zip(model.named_parameters(), ref.parameters()):
    c.check(f"grad {n}", torch.allclose(p.grad, q.grad, rtol=1e-5, atol=1e-6),
            f"max diff {float((p.grad - q.grad).abs().max())}")
c.finish()
