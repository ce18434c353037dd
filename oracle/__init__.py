"""Test-only CPU oracle for the Flash-KMeans Lloyd hot path (see kmeans_oracle)."""
