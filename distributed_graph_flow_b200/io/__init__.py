"""GF graph loading: raw-id mapping on the device, Parquet shards on the host."""
