"""Link-prediction example generation (positive and negative node pairs)."""
