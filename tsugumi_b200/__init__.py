"""tsugumi_b200: Tsugumi's MoE feed-forward block for B200 (sm_100a).

The compute lives in libtsugumi_cuda.so (hand-written CUDA + a C ABI,
include/tsugumi_cuda.h); this package holds its build script, the ctypes
bindings, the host-side mirror of the reference's encoder classes, the
.moepack packed-experts reader (moepack.py), and the seeded synthetic-layer
generator used by the tests and the benchmark.
"""

from ._abi import TsgError  # noqa: F401
from .moe import (  # noqa: F401
    Context,
    MoE,
    MoELayer,
    PrefillGroupedRoutedMoE,
    PrefillMoE,
    PrefillMoEGrouping,
    PrefillMoEGroupingError,
    PrefillRoutedGEMMPlanner,
    PrefillRouter,
    SharedExpertRuntime,
    last_routing,
)


def upload_host_layer(host, device: int = 0) -> dict:
    """Device tensors (torch) for a synthetic.HostLayer, in the blob format."""
    import torch

    dev = torch.device("cuda", device)
    t = {
        "d": host.d, "f": host.f, "num_experts": host.num_experts, "top_k": host.top_k,
        "act": host.act, "experts": torch.from_numpy(host.experts).to(dev),
        "expert_stride": host.expert_stride, "offsets": host.offsets,
        "router_w": torch.from_numpy(host.router_w).to(dev),
    }
    if host.shared is not None:
        t.update(shared=torch.from_numpy(host.shared).to(dev), shared_f=host.shared_f,
                 shared_offsets=host.shared_offsets)
        if host.shared_gate is not None:
            t["shared_gate"] = torch.from_numpy(host.shared_gate).to(dev)
    if host.logit_bias is not None:
        t["logit_bias"] = torch.from_numpy(host.logit_bias).to(dev)
    return t
