"""Multi-GPU components: failure-agreement transport (:mod:`.distributed`), tiered sequence-parallel
KV history (:mod:`.sp_kv`), factor sharding (:mod:`.factor_sharding`) and context parallelism
(:mod:`.context_parallel`)."""
