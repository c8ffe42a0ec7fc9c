"""An ordinary PyTorch training script with no fault-tolerance code in it;
the transparent-mode test runs it unchanged under the harness."""
import os

import torch

torch.manual_seed(0)
model = torch.nn.Sequential(torch.nn.Linear(16, 64), torch.nn.ReLU(), torch.nn.Linear(64, 1))
opt = torch.optim.AdamW(model.parameters(), lr=1e-2, weight_decay=0.01)
data = torch.Generator().manual_seed(1000 + int(os.environ.get("SHIFT_REPLICA_ID", "0")))
step = 0
while True:
    x = torch.randn(32, 16, generator=data)
    y = x.sum(1, keepdim=True).tanh()
    opt.zero_grad()
    loss = ((model(x) - y) ** 2).mean()
    loss.backward()
    opt.step()
    step += 1
