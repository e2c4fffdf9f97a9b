"""GPU operators: thin Python wrappers over the sm_100a extension plus plain-PyTorch
reference implementations of the same math (used as CPU oracles and on CPU tensors)."""
