"""Data: synthetic batches, GPIC webdataset shards with the cached text-encoder outputs, crops, length buckets."""
