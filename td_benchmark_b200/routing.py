"""On-device routing ahead of the layer: gate GEMM -> softmax -> top-k -> renormalise.

The reference routes on its data-preparation side, outside the timed layer
(``moe_bench/data/routing.py:49-74``, ``moe_bench/worker.py:205-208``): every rank takes
``hidden_local.float() @ gate_weight.float().T`` (fp32), adds ``strength * log(E * p)``
under imbalanced routing (``routing.py:59-61``), takes softmax -> top-k -> renormalise and
all-gathers the ids and weights so every rank holds the routing of all T tokens.

``Router`` runs the same steps on the device with buffers sized once:

* the gate GEMM is a plain fp32 GEMM and goes to cuBLAS (``torch.matmul`` into a
  preallocated buffer), the library call the reference's own ``@`` makes;
* ``b2m_route_topk`` fuses the bias add, softmax, top-k and renormalisation;
* with several ranks, ``all_gather_into_tensor`` of the ids and weights (8 bytes per
  (token, expert) pair -- 0.5 MB for the DeepSeek-V3 layer).

``router(x_local)`` returns ``(topk_ids [T, k] int32, topk_weights [T, k] fp32)`` for all
T tokens, ready for ``MoELayer.forward``.
"""
from __future__ import annotations

import torch

from . import ops
from .configs import RoutingCfg


def log_prior(cfg: RoutingCfg, experts: int, device) -> torch.Tensor | None:
    """``strength * log(E * p)`` for the routing's target distribution p, None when uniform."""
    if cfg.imbalance_kind == "none":
        return None
    from .data import target_distribution

    # computed on the host, like the reference's bundle on CPU, then moved: the same bits on every device
    p = target_distribution(cfg, experts)
    return (cfg.strength * torch.log(experts * p)).to(torch.float32).to(device).contiguous()


class Router:
    def __init__(self, gate_weight: torch.Tensor, tokens_local: int, top_k: int, bias: torch.Tensor | None = None,
                 group=None, device=None):
        """gate_weight [E, H] (any float dtype); tokens_local = this rank's token count."""
        self.device = torch.device(device) if device is not None else gate_weight.device
        self.gate_t = gate_weight.to(self.device, torch.float32).t().contiguous()   # [H, E]
        self.experts = gate_weight.shape[0]
        self.top_k = top_k
        self.bias = None if bias is None else bias.to(self.device, torch.float32).contiguous()
        self.group = group
        self.world = 1
        if group is not None or (torch.distributed.is_available() and torch.distributed.is_initialized()):
            self.world = torch.distributed.get_world_size(group)
        dev = self.device
        H = gate_weight.shape[1]
        self.x32 = torch.empty((tokens_local, H), dtype=torch.float32, device=dev)
        self.logits = torch.empty((tokens_local, self.experts), dtype=torch.float32, device=dev)
        self.ids_local = torch.empty((tokens_local, top_k), dtype=torch.int32, device=dev)
        self.w_local = torch.empty((tokens_local, top_k), dtype=torch.float32, device=dev)
        if self.world > 1:
            self.ids = torch.empty((tokens_local * self.world, top_k), dtype=torch.int32, device=dev)
            self.w = torch.empty((tokens_local * self.world, top_k), dtype=torch.float32, device=dev)
        else:
            self.ids, self.w = self.ids_local, self.w_local

    def __call__(self, x_local: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        self.x32.copy_(x_local)
        torch.matmul(self.x32, self.gate_t, out=self.logits)
        ops.route_topk(self.logits, self.top_k, self.bias, out=(self.ids_local, self.w_local))
        if self.world > 1:
            import torch.distributed as dist
            dist.all_gather_into_tensor(self.ids, self.ids_local, group=self.group)
            dist.all_gather_into_tensor(self.w, self.w_local, group=self.group)
        return self.ids, self.w
