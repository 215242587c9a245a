"""Token-shard preparation (``prepare_data``, ``build_small_shard``)."""
