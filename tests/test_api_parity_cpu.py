"""API parity with the reference, checked without its source tree: every public class and function of each reference
module is reachable from the module that replaces it here, and every command-line flag of the reference's training,
chat, serving, fine-tuning, distillation, benchmark and sampling scripts is accepted by the matching tool. The name
and flag lists below were read off the reference's modules (``src/*.py``); they are its interface, kept as data."""

import argparse
import importlib

import pytest

# (reference module, modules here that together provide its names, the reference module's public names)
MODULES = [('fast_decode', 'inference.fast_decode',
  ['FastDecoder', 'Unsupported', 'capture_mode', 'filter_logits', 'layer_weight', 'precision_dtype']),
 ('quantization', 'inference.quantization',
  ['QuantizedLinear', 'load_quantized', 'quantize_model', 'save_quantized']),
 ('lora', 'tools.lora',
  ['LoRALinear', 'adapter_state', 'add_lora', 'load_adapter', 'merge_lora_state', 'save_adapter']),
 ('expert_parallel', 'parallel.expert_parallel parallel.checkpoint',
  ['DeviceLoadTracker', 'ExpertParallelContext', 'ExpertParallelMoE', 'all_reduce_mean', 'barrier',
   'broadcast_shared_parameters', 'clip_grad_norm_parallel', 'consolidate_checkpoint', 'finish',
   'init_expert_parallel', 'is_expert_parameter', 'load_sharded_checkpoint', 'reshard_checkpoint',
   'save_sharded_checkpoint', 'shard_path', 'sharded_checkpoint_exists', 'sync_gradients']),
 ('tensor_parallel', 'parallel.tensor_parallel',
  ['TensorParallelAttention', 'copy_to_tp', 'is_tp_sharded', 'is_tp_sharded_shared', 'merge_state_dicts',
   'merge_tensors', 'reduce_from_tp', 'shard_state_dict', 'shard_tensor']),
 ('pipeline_parallel', 'parallel.pipeline_parallel',
  ['PipelineContext', 'PipelineEngine', 'clip_grad_norm_pipeline', 'init_pipeline_parallel', 'partition_layers']),
 ('sharded_optimizer', 'parallel.sharded_optimizer', ['ShardedAdamW']),
 ('data_pipeline', 'data.pipeline',
  ['BPETokenizer', 'BatchStream', 'CharTokenizer', 'CharacterDataset', 'CurriculumConfig', 'DomainMixture',
   'Segment', 'SentencePieceTokenizer', 'TokenCorpus', 'WindowDataset', 'build_corpus', 'difficulty_scores',
   'extract_text', 'load_token_bin', 'load_tokenizer', 'parse_domain_weights', 'read_rows', 'token_classes',
   'write_token_bin']),
 ('moe_schedules', 'training.schedules', ['ScheduleConfig', 'TrainingController', 'schedule_field_names']),
 ('training_metrics', 'training.metrics', ['MetricsLogger', 'detect_plateau', 'first_stable_step']),
 ('routing_diagnostics', 'utils.routing_diagnostics',
  ['RoutingMonitor', 'bar_chart_svg', 'heatmap_svg', 'line_chart_svg']),
 ('run_bundle', 'tools.run_bundle',
  ['add_archive_arguments', 'archive_data', 'create_run_bundle', 'environment_info', 'epoch_folder',
   'reproduce_command', 'resolve_archive_dir', 'run_benchmarks', 'write_held_out_sample', 'write_samples']),
 ('experiment_manager', 'tools.experiment_manager',
  ['bar_chart_svg', 'compare_pareto', 'compare_runs', 'dig', 'dominates', 'git_revision', 'load_config',
   'load_summaries', 'loss_curves_svg', 'main', 'objective_of', 'pareto_front', 'parse_objectives',
   'render_run_report', 'run_experiment', 'run_final_benchmark', 'slug', 'update_best']),
 ('sweep', 'tools.sweep',
  ['expand_grid', 'invalid_reason', 'main', 'make_experiment', 'run_bayes_sweep', 'run_bohb_sweep', 'run_sweep',
   'sample_random', 'sample_value']),
 ('bayes_opt', 'tools.bayes_opt',
  ['BayesianOptimizer', 'GaussianProcess', 'SearchSpace', 'expected_improvement', 'matern52']),
 ('hardware', 'utils.hardware',
  ['DeviceInfo', 'auto_architecture', 'choose_precision', 'detect', 'find_safe_batch_size', 'main',
   'parameter_counts', 'recommend', 'suggest_num_experts', 'training_state_bytes']),
 ('energy_tracking', 'utils.energy', ['PowerCostTracker']), ('pii_redact', 'utils.pii_redact', ['PIIRedactor']),
 ('cross_tokenizer', 'tools.cross_tokenizer',
  ['CrossTokenizerLoss', 'HFTeacher', 'align_positions', 'first_char_matrix', 'marginal_kl', 'student_pieces',
   'uld_loss']),
 ('distill_quantweave_moe', 'tools.distill',
  ['build_parser', 'distillation_loss', 'load_model', 'main', 'run_distillation']),
 ('finetune_quantweave_moe', 'tools.finetune',
  ['build_parser', 'evaluate', 'load_base', 'load_finetuned', 'main', 'run_finetune']),
 ('chat_quantweave_moe', 'tools.chat',
  ['ChatSession', 'Reply', 'Settings', 'apply_setting', 'build_parser', 'choose_token', 'load_for_chat', 'main',
   'read_messages', 'repl', 'resolve_model', 'run_batch', 'run_folders', 'usable_model']),
 ('serve_quantweave', 'tools.serve',
  ['ChatMessage', 'ChatRequest', 'GenerateRequest', 'JSONLogFormatter', 'Metrics', 'Moderation', 'RateLimiter',
   'Server', 'build_app', 'build_parser', 'configure_logging', 'main', 'reply_payload']),
 ('export_quantweave', 'tools.export',
  ['LogitsOnly', 'export_bundle', 'load_checkpoint_model', 'load_exported', 'main', 'parity_shapes', 'sha256',
   'try_onnx']),
 ('benchmark_quantweave_moe', 'tools.benchmark',
  ['build_parser', 'histogram', 'main', 'process_rss_bytes', 'render_markdown', 'routing_and_compute',
   'run_benchmark', 'synchronize', 'training_stability']),
 ('generate_quantweave_moe', 'tools.generate', ['main', 'sample_text']),
 ('cpu_offload_optimizer', 'optim.cpu_offload', ['CPUOffloadAdamW']),
 ('checkpoint_io', 'utils.checkpoint_io', ['load_checkpoint']),
 ('model_scaling', 'tools.model_scaling', ['ModelSpec', 'billions', 'load_presets', 'main', 'make_spec']),
 ('prepare_tokens', 'tools.prepare_tokens', ['main']),
 ('train_quantweave_moe', 'training.trainer',
  ['autocast_context', 'build_optimizer', 'build_parser', 'build_vocab', 'checkpoint_exists', 'config_hash',
   'default_args', 'diff_fields', 'evaluate_validation', 'load_checkpoint', 'load_data', 'main', 'restore_rng',
   'resume_fields', 'run_training', 'save_checkpoint', 'schedule_config_from', 'select_device', 'tokenizer_hash',
   'tokenizer_payload', 'write_checkpoint_metadata']),
 ('moe_kernels', 'moe_kernels',
  ['GroupedPlan', 'benchmark', 'compute_dtype', 'experts_support_grouped', 'grouped_matmul', 'grouped_swiglu',
   'kernels_available']),
 ('quantweave_moe_model', 'models.model models.moe config',
  ['QuantaWeaveBlock', 'QuantaWeaveConfig', 'QuantaWeaveMoEForCausalLM', 'SparseSwiGLU', 'TopKMoE'])]

# reference script -> its command-line flags
FLAGS = {'benchmark_quantweave_moe': ['--batch-size', '--checkpoint', '--data', '--device', '--examples',
                              '--no-routing-stats', '--output', '--precision', '--training-metrics'],
 'chat_quantweave_moe': ['--adapter', '--checkpoint', '--conversation', '--device', '--interactive', '--json',
                         '--latest', '--messages-file', '--mode', '--no-cache', '--precision', '--quantize',
                         '--quiet', '--run', '--runs-dir', '--seed', '--stop', '--system', '--temperature',
                         '--tokens', '--top-k', '--top-p', '--transcript'],
 'distill_quantweave_moe': ['--alpha', '--batch-size', '--checkpoint-dir', '--checkpoint-interval', '--cross-loss',
                            '--device', '--examples', '--hf-teacher', '--lr', '--output', '--precision', '--resume',
                            '--seed', '--sequence-length', '--steps', '--student', '--teacher-checkpoint',
                            '--teacher-data', '--temperature'],
 'finetune_quantweave_moe': ['--alpha', '--batch-size', '--bits', '--checkpoint', '--data', '--device',
                             '--examples', '--group-size', '--include-lm-head', '--lr', '--merge-output',
                             '--optimizer', '--output', '--precision', '--rank', '--seed', '--sequence-length',
                             '--steps', '--train-norms', '--train-router'],
 'generate_quantweave_moe': ['--checkpoint', '--device', '--precision', '--prompt', '--temperature', '--tokens'],
 'serve_quantweave': ['--adapter', '--api-key', '--checkpoint', '--device', '--host', '--latest', '--log-format',
                      '--max-queue', '--moderation-blocklist', '--no-cache', '--port', '--precision',
                      '--rate-limit', '--rate-limit-window', '--request-timeout', '--run', '--runs-dir'],
 'train_quantweave_moe': ['--activation-checkpointing', '--active-experts', '--allow-config-change',
                          '--archive-benchmark-examples', '--archive-data-limit-mb', '--archive-dir',
                          '--attention-heads', '--auto-architecture', '--auto-architecture-memory-fraction',
                          '--auto-architecture-quality', '--auto-batch-size', '--auto-batch-target', '--aux-adapt',
                          '--aux-coef-end', '--batch-size', '--capacity-adapt', '--capacity-factor',
                          '--capacity-max', '--capacity-min', '--capacity-release-step', '--checkpoint-dir',
                          '--checkpoint-interval', '--controller-interval', '--curriculum',
                          '--curriculum-start-fraction', '--curriculum-steps', '--data', '--data-card', '--device',
                          '--device-metrics', '--diagnostics-dir', '--diagnostics-interval',
                          '--domain-specialization-coef', '--domain-weights', '--domain-weights-end',
                          '--domain-weights-steps', '--drop-overflow-tokens', '--drop-threshold',
                          '--electricity-rate-usd-kwh', '--examples', '--expert-parallel', '--ffn-size',
                          '--gradient-accumulation-steps', '--hidden-size', '--layers', '--log-interval', '--lr',
                          '--lr-decay', '--metrics-file', '--microbatches', '--min-expert-capacity',
                          '--min-lr-ratio', '--moe-kernel', '--no-archive', '--no-power-tracking', '--optimizer',
                          '--output', '--overflow-policy', '--pipeline-parallel', '--pipeline-schedule',
                          '--plateau-patience', '--precision', '--redact-pii', '--resume', '--router-aux-coef',
                          '--router-temperature', '--schedule-steps', '--seed', '--sequence-length',
                          '--shard-optimizer', '--simulate-slow-rank', '--steps', '--straggler-capacity',
                          '--straggler-capacity-max', '--straggler-capacity-min', '--straggler-interval',
                          '--straggler-max-bias', '--straggler-routing', '--straggler-strength',
                          '--temperature-adapt', '--temperature-start', '--temperature-steps', '--tensor-parallel',
                          '--token-data', '--tokenizer', '--tokenizer-algorithm', '--tokenizer-path',
                          '--total-experts', '--val-batches', '--val-fraction', '--val-interval', '--val-seed',
                          '--vocab-size', '--warmup-steps']}

TOOLS = {
    "train_quantweave_moe": "training.trainer", "chat_quantweave_moe": "tools.chat", "serve_quantweave": "tools.serve",
    "finetune_quantweave_moe": "tools.finetune", "distill_quantweave_moe": "tools.distill",
    "benchmark_quantweave_moe": "tools.benchmark", "generate_quantweave_moe": "tools.generate",
}


@pytest.mark.parametrize("reference,ours,names", MODULES, ids=[m[0] for m in MODULES])
def test_every_public_name_of_the_reference_module_exists(reference, ours, names):
    modules = [importlib.import_module("quantaweave_b200." + m) for m in ours.split()]
    missing = [n for n in names if not any(hasattr(m, n) for m in modules)]
    assert not missing, (reference, missing)


def _flags(parser: argparse.ArgumentParser) -> set:
    out = set()
    for action in parser._actions:
        if isinstance(action, argparse._SubParsersAction):
            for sub in action.choices.values():
                out |= _flags(sub)
        out |= set(action.option_strings)
    return out


@pytest.mark.parametrize("script", sorted(FLAGS))
def test_every_flag_of_the_reference_script_is_accepted(script):
    parser = importlib.import_module("quantaweave_b200." + TOOLS[script]).build_parser()
    missing = sorted(set(FLAGS[script]) - _flags(parser))
    assert not missing, (script, missing)
