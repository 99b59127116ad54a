"""moe_b200 — B200 (sm_100a) MoE-layer hot path of naiwa-rs behind its operator interface.

`RoutedExpertsProvider.build(ctx)` / `RoutedExperts.forward(xs, topk_weights, topk_ids)` mirror
the reference's fork traits (naiwa-rs src/moe/provider.rs:316-615, src/moe/cached_layer.rs:524-664,
src/moe/expert.rs:59-117); `route` is the router + top-k upstream of them. All compute runs in
libmoe_b200.so; torch tensors are only the containers for device memory and streams.
"""
from ._lib import (  # noqa: F401
    DTYPE_BF16, DTYPE_FP8_E4M3_B128, DTYPE_Q2_0, DTYPE_Q4_K, DTYPE_Q8_0, MOE_ID_NONE, MoeError, ROUTER_SIGMOID_GROUP,
    ROUTER_SOFTMAX, ROUTER_SOFTMAX_RENORM, lib,
)
from .layer import (  # noqa: F401
    ExpertLoadContext, MoeConfig, RoutedExperts, RoutedExpertsProvider, Router, plan_pairs, requantize_q2_0,
    route_tokens,
)
from .ep import ExpertParallelMoE, PeerExpertParallelMoE, ep_combine, ep_dispatch, ep_pack_rows  # noqa: F401,E402
from .doorbell import Ring  # noqa: F401,E402
from .cpu import CpuExperts, Executor, add_f32_into_bf16, cpu_isa  # noqa: F401,E402
from .paged import PagedMoE  # noqa: F401,E402
from .gguf import GGUFFile  # noqa: F401,E402
