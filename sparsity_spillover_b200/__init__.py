"""B200-native (sm_100a) activation-sparse GPT-NeoX MLP forward.

A drop-in for the reference's gated MLP hot path (thiagocmattar/sparsity-spillover):

* ``ops``       tensor-level entry points over the C ABI of ``libspmlp.so``
                (``include/spmlp.h``) and ``torch.ops.spmlp.*`` registrations;
* ``mlp``       ``SparseGPTNeoXMLP`` / ``SparseHead`` modules, ``install(model)``, the
                joint consumer ``JointConsumer`` and ``install_joint(model)``, the head
                installer ``install_head(model, mode, config)``;
* ``gates``     the reference's gate specs and modules -> kernel gate enum;
* ``workloads`` seeded synthetic inputs of the benchmark configs;
* ``dist``      token sharding and the d_ff split (NCCL collectives, and the fused
                form whose down projection stores partial tiles into peer memory);
* ``pipeline``  a multi-layer stack with host-to-host streaming;
* ``measurement`` the reference harness's paired, rotating-input timing protocol.

Every compute call goes through libspmlp.so; there is no CPU fallback.
"""
from __future__ import annotations

__all__ = ["ops", "mlp", "gates", "workloads", "SparseGPTNeoXMLP", "SparseHead", "install", "JointConsumer",
           "install_joint", "install_head"]


def __getattr__(name):
    if name in ("SparseGPTNeoXMLP", "SparseHead", "install", "JointConsumer", "install_joint", "install_head"):
        from . import mlp

        return getattr(mlp, name)
    if name in ("ops", "mlp", "gates", "workloads", "dist"):
        import importlib

        return importlib.import_module(f".{name}", __name__)
    raise AttributeError(name)
