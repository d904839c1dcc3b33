"""Host-side compression metadata: selection, query window, events, blocks."""
