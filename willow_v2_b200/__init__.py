"""willow_v2_b200: a B200-native (sm_100a) implementation of willow's qwen35moe MoE block.

The CUDA kernels and the C ABI live in csrc/ and are built into libwmoe.so (see willow_v2_b200.build).
Python-side pieces: lib (ctypes binding of the C ABI), store (the HBM expert store), moe (the Engine.moe
drop-in), synth (seeded synthetic inputs), ep (expert parallelism over torch.distributed/NCCL)."""
