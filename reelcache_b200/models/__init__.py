"""From-scratch video DiTs on the sm_100a kernels: the CausVid-shaped causal Wan DiT
(:mod:`.causal_wan`) with its DMD chunk sampler (:mod:`.sampler`), its FP32 reference
(:mod:`.reference`), and the LongCat-shaped DiT (:mod:`.longcat`)."""
