"""TEST INFRASTRUCTURE ONLY: CPU restatements of TVdxSampler used as the parity checker."""
