# Entry points by name (the same target names as gpt2-harness where the
# capability exists). Every target runs a module of this package; results go
# under results/, figures under figures/.

PY ?= python
NPROC ?= 8
TORCHRUN = $(PY) -m torch.distributed.run --nnodes=1 --nproc-per-node $(NPROC) --master-addr 127.0.0.1

.PHONY: help build test test-fast gpu-test verify ablate induction kv quantize prune distill \
        parallel roofline diagnose cluster collectives preflight dry-run smoke bench bench-scaling \
        bench-ref baseline-ref compare figures all clean

help:
	@grep -E '^[a-z-]+:.*?## ' $(MAKEFILE_LIST) | sed 's/:.*## /\t/'

build: ## compile the sm_100a extension in-tree
	$(PY) setup.py build_ext --inplace

test: ## CPU tier (oracle strategies over gloo, host orchestration, launchers)
	$(PY) -m pytest tests -q -m "not gpu"

test-fast: ## CPU tier without the multi-process tests marked slow
	$(PY) -m pytest tests -q -m "not gpu and not slow"

gpu-test: ## B200 tier (kernels against fp32 torch, native strategies against one GPU)
	$(PY) -m pytest tests -q -m gpu

verify: ## oracle model against a local HF checkpoint
	$(PY) -m gpt2_harness_b200.experiments verification --out results

ablate: ## 9 architecture arms x 3 seeds
	$(PY) -m gpt2_harness_b200.experiments ablations --out results

induction: ## induction-head scores and ablations
	$(PY) -m gpt2_harness_b200.experiments induction --out results

kv: ## cached vs uncached decoding
	$(PY) -m gpt2_harness_b200.experiments kv_cache --out results

quantize: ## int8/int4 weight quantisation sweep
	$(PY) -m gpt2_harness_b200.experiments quantization --out results

prune: ## head / neuron pruning sweep
	$(PY) -m gpt2_harness_b200.experiments pruning --out results

distill: ## student distillation
	$(PY) -m gpt2_harness_b200.experiments distillation --out results

parallel: ## every strategy's equivalence and closed-form payload check (gloo)
	$(PY) -m gpt2_harness_b200.parallel.run_parallel --out results

roofline: ## measured peaks, per-op roofline, per-kernel and per-strategy fractions
	$(PY) -m gpt2_harness_b200.perf.roofline
	$(PY) -m gpt2_harness_b200.perf.path_roofline

diagnose: ## step breakdown and ranked findings
	$(PY) -m gpt2_harness_b200.perf.diagnose

cluster: ## checkpoint resharding, streaming, kill-and-restart
	$(PY) -m gpt2_harness_b200.cluster.run_cluster --out results

collectives: ## all-reduce / all-gather / reduce-scatter sweep (NCCL and the P2P kernel)
	$(PY) -m gpt2_harness_b200.cluster.collbench --world $(NPROC) --max-mib 256

preflight: ## placement, backend and precision decisions on this machine
	$(PY) -m gpt2_harness_b200.preflight

dry-run: ## the same decisions on a fabricated 8 x B200 node
	$(PY) -m gpt2_harness_b200.preflight --dry-run --stub-gpus 8

smoke: ## one tiny forward + backward on cuda:0
	$(PY) -c "import __graft_entry__ as g; g.smoke(); print('smoke ok')"

bench: ## headline benchmark, one GPU
	$(PY) bench.py

bench-scaling: ## headline benchmark on NPROC GPUs
	$(TORCHRUN) bench.py --gpus $(NPROC)

REF_SRC ?= ../reference
baseline-ref: ## install the unmodified reference into baseline/_ref (offline, from REF_SRC)
	rm -rf /tmp/g2b_ref_src && cp -r $(REF_SRC) /tmp/g2b_ref_src
	$(PY) -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse \
	    --target baseline/_ref --upgrade /tmp/g2b_ref_src
	test -d baseline/_ref/transformer_internals

bench-ref: ## the reference arm of the headline benchmark, one GPU
	$(PY) bench.py --impl reference

compare: ## gate a results tree against the committed one
	$(PY) -m gpt2_harness_b200.compare_results --baseline-git HEAD --current results

figures: ## redraw every figure from results JSON
	$(PY) -m gpt2_harness_b200.experiments figures --out results --figures figures

all: test parallel cluster figures

clean:
	rm -rf build
