"""Engine-side pieces of the attention hot path (mirrors the reference's
``engine`` package for the modules the path touches: ``engine.attention`` and
``engine.cache``), plus the kv-head sharding layer ``engine.head_shard``."""
