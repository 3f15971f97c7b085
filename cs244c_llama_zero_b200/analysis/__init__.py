"""Reports and charts over experiment run directories (summary.json, tuning_summary.json, profile JSON)."""
