"""Parallelism: ZeRO-1/2 data parallel, tensor/sequence parallel, 1F1B pipeline parallel."""
