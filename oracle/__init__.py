"""CPU restatement of the reference's bucketMul decode path: test infrastructure only."""
