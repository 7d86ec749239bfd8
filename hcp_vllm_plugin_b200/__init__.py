"""B200-native (sm_100a) ring context-parallel attention for vLLM.

Drop-in for the reference plugin's hot path (stark-sim/hcp-vllm-plugin):
``register()`` installs the same names with vLLM - the ``CUSTOM`` attention
backend ``HcpRingAttentionBackend`` and the ``HcpRingKvConnector`` /
``HcpFileConnector`` KV connectors (``hcp_vllm_plugin/__init__.py:34-54``) -
and the attention math runs in ``libhcp_ring.so`` (hand-written tcgen05/TMA
CUDA behind a C ABI, ``include/hcp_ring.h``).
"""

__version__ = "0.1.0"


def register() -> None:
    """vLLM ``general_plugins`` entry point: register backend and connectors."""
    from vllm.distributed.kv_transfer.kv_connector.factory import KVConnectorFactory
    from vllm.v1.attention.backends.registry import AttentionBackendEnum, register_backend

    registry = getattr(KVConnectorFactory, "_registry", {})
    if "HcpRingKvConnector" not in registry:
        KVConnectorFactory.register_connector(
            "HcpRingKvConnector", "hcp_vllm_plugin_b200.ring_connector", "HcpRingKvConnector")
    if "HcpFileConnector" not in registry:
        KVConnectorFactory.register_connector(
            "HcpFileConnector", "hcp_vllm_plugin_b200.file_connector", "HcpFileConnector")
    register_backend(
        AttentionBackendEnum.CUSTOM,
        "hcp_vllm_plugin_b200.ring_backend.HcpRingAttentionBackend",
    )
