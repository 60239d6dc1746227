"""STD (sparse-to-dense self-speculative decoding) hot path on B200 / sm_100a."""
