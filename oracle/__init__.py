"""CPU oracle package: a restatement of squirrel-rs's token loop used only to check the GPU path."""
