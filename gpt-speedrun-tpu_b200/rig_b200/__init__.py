"""rig_b200 — B200-native drop-in for the GPT-speedrun rig's training-step path.

Mirrors the reference plugin surface (`rig.nn`, `rig.attention`,
`rig.kernels`, `rig.mesh`, `rig.tokens`) on top of libgptb200.so, the C ABI of
hand-written sm_100a kernels declared in include/gptb200.h. `model.GPTTrainer`
is the whole training step.
"""

__version__ = "0.1.0"
