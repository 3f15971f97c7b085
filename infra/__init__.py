"""Host-side infrastructure: the LD_PRELOAD socket shaper and its builder, tc / launch / setup scripts."""
