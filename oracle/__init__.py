"""CPU checkers for the flat PQ search path — TEST INFRASTRUCTURE ONLY.

`oracle.port` wraps the plain-C restatement (vk_oracle.c) of the reference CPU path; `oracle.ref` wraps the
reference's own CPU library compiled from its sources (present only where the reference was available at build
time). Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this package, and only to
check or time the CPU path; the product (veckern_b200) never does.
"""
from .oracle import Port, Ref, port, ref, ref_available  # noqa: F401
