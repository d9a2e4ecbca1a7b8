"""Event ingest for the B200 forward (cortex/data in the reference)."""

from cortex.data.ingest import (PackedBatch, bucket_values, collate_events, collate_windows,
                                events_from_bin_matrix)

__all__ = ["PackedBatch", "bucket_values", "collate_events", "collate_windows",
           "events_from_bin_matrix"]
