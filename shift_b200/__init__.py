"""shift_b200: a B200-native fault-tolerant MoE training harness.

Layers (bottom to top): sm_100a kernels (``ops``), model (``models``),
parallel layers and collectives (``parallel``), the fault-tolerance control
plane (``ft``: lighthouse, manager, transport, handoff protocols), node and
cluster control (``control``) and offline evidence analysis (``analysis``).
"""
__version__ = "0.1.0"
