"""rai_b200: B200-native (sm_100a) prompt-lookup speculative decode step for
rai-infer .raimodel models, behind a C ABI (include/rai_gpu.h)."""
from .api import (LookupConfig, LookupDecoder, LookupMetrics, RaiError, RaiModel, SpeculativeDecoder,  # noqa: F401
                  StepBatch, prefill_many, step_many)
