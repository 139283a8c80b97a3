"""Oracle package: CPU restatement of the reference path, and the reference's own
CPU evaluator built into ``oracle/_ref``. Test infrastructure only; the product
never imports it."""
