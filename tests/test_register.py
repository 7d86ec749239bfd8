"""The vLLM plugin entry point installs the reference's names
(``hcp_vllm_plugin/__init__.py:34-54``) and every name resolves to a class
of this package."""


def test_register_installs_backend_and_connectors():
    from vllm.distributed.kv_transfer.kv_connector.factory import KVConnectorFactory
    from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorBase_V1
    from vllm.v1.attention.backends.registry import AttentionBackendEnum

    from hcp_vllm_plugin_b200 import register
    from hcp_vllm_plugin_b200.file_connector import HcpFileConnector
    from hcp_vllm_plugin_b200.ring_backend import HcpRingAttentionBackend
    from hcp_vllm_plugin_b200.ring_connector import HcpRingKvConnector

    register()
    register()  # idempotent
    assert AttentionBackendEnum.CUSTOM.get_path() == "hcp_vllm_plugin_b200.ring_backend.HcpRingAttentionBackend"
    assert AttentionBackendEnum.CUSTOM.get_class() is HcpRingAttentionBackend
    assert HcpRingAttentionBackend.get_name() == "CUSTOM"
    assert HcpRingAttentionBackend.forward_includes_kv_cache_update is False
    for name, cls in (("HcpRingKvConnector", HcpRingKvConnector), ("HcpFileConnector", HcpFileConnector)):
        got = KVConnectorFactory.get_connector_class_by_name(name)
        assert got is cls and issubclass(got, KVConnectorBase_V1)
