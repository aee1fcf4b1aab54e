"""The callers of the op: workloads and their input tensors, drivers and timers, the
multi-layer decode step and the per-GPU shards.

configs     Workload (one call's shape, its layout variants, how it shards) and the five B200
            workloads
inputs      the tensors of one call for a Workload
positions   device-resident position sets for timed loops
runners     eager and graph-bound drivers of a stream of calls
timing      byte accounting (the roofline numerator) and the per-call timer
decode_loop the 32-layer decode step captured as one CUDA graph
sharding    per-GPU slices of a call and the harness-side gather
"""
