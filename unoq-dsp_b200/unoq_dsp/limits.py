"""Plan contract bounds, identical to the reference runtime (runtime/graph.h:5-9, qnn.h:10-11)."""
MAX_TENSORS = 1024
MAX_OPERATORS = 512
ARENA_BYTES = 16 * 1024 * 1024
MAX_PLAN_BYTES = 17 * 1024 * 1024
MAX_WORK = 2_000_000_000
MAX_CHANNELS = 2048
