"""ugdr-b200: a userspace GPU RDMA (verbs) library for 8xB200 NVLink 5 / NVSwitch nodes.

Layout:
  verbs      Pythonic wrappers over the C verbs ABI (libugdr.so) and the daemon launcher
  ops        device kernels callable from Python (copy core, collective kernels)
  parallel   collectives on registered memory: allreduce (fused bf16 sum), MoE all-to-all
  models     workload definitions: the benchmark configurations and the MoE router
  utils      build, timing and clock-sampling helpers
"""
__version__ = "0.1.0"
