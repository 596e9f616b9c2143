"""CPU oracle of the Qwen3-MoE expert path -- test infrastructure only.

``moe_oracle``: numpy / torch-CPU restatement of the reference algorithm,
pinned against golden vectors from the reference (tests/golden).
``cpu_ops``: the kernel interface implemented with the oracle on CPU tensors,
for exercising host logic without a GPU.
"""
