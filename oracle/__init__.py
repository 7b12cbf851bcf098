"""CPU checkers for the flat PQ search path — TEST INFRASTRUCTURE ONLY.

`oracle.port` wraps the plain-C restatement (vk_oracle.c) of the reference CPU path; `oracle.ref` wraps the
reference's own CPU library compiled from its sources (present only where the reference was available at build
time). `oracle.inputs` restates the configurations' input generators in numpy, and `oracle.refgpu_sweep` runs the
reference's own GPU kernel, both for bench.py's reference arm. Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg and reference arm import this package, and only to check or time the reference; the product
(veckern_b200) never does.
"""
from .oracle import Port, Ref, port, ref, ref_available, refgpu_available, refgpu_sweep  # noqa: F401
