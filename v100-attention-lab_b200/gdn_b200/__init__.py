"""gdn_b200 -- B200-native chunked Gated DeltaNet forward (sm_100a).

Drop-in for the forward entry point of 123123213weqw/v100-attention-lab
(``gdn_triton.gdn_chunk_fwd``); see ``ops.gdn_chunk_fwd``.
"""

from .fla_compat import chunk_delta_rule, chunk_gated_delta_rule
from .ops import GdnError, check_status, gdn_chunk_fwd, gdn_chunk_fwd_fixed, gdn_chunk_fwd_v2, gdn_wy_prep

__all__ = ["gdn_chunk_fwd", "gdn_chunk_fwd_v2", "gdn_chunk_fwd_fixed", "gdn_wy_prep", "chunk_gated_delta_rule",
           "chunk_delta_rule", "GdnError", "check_status"]
