// zealot_rl_ffi.rs -- the Rust declarations of include/zealot_rl.h, one per
// entry point, for the zealot-rl-cuda crate (zealot-rl-cuda/src/ffi.rs).
// Written against the header; no Rust toolchain builds it here, and
// tests/test_ffi_decls.py keeps its entry points, argument and return types
// (pointee constness included) and struct fields equal to the header's.
use std::os::raw::{c_char, c_int, c_void};

#[repr(C)] pub struct ZrlCtx { _p: [u8; 0] }
#[repr(C)] #[derive(Clone, Copy)]
pub struct ZrlPpoConfig {            // PpoConfig (ppo.rs:22-65)
    pub gamma: f32, pub lam: f32, pub clip: f32, pub entropy_coef: f32,
    pub value_coef: f32, pub epochs: i32, pub minibatches: i32,
    pub max_grad_norm: f32, pub desired_kl: f32, pub lr_min: f32,
    pub lr_max: f32, pub adaptive_lr: i32,
}
#[repr(C)] #[derive(Clone, Copy, Default)]
pub struct ZrlStats { pub kl: f32, pub surrogate: f32, pub value_loss: f32,
                      pub entropy: f32, pub lr: f32 }   // PpoStats
#[repr(C)]
pub struct ZrlModelConfig { pub n_actor_dims: i32, pub actor_dims: [i32; 9],
                            pub n_critic_dims: i32, pub critic_dims: [i32; 9],
                            pub max_samples: i64, pub precision: i32 }
#[repr(C)]
pub struct ZrlComm { pub rank: i32, pub world_size: i32,
                     pub nccl_id: [u8; 128], pub timeout_ms: i32 }
#[repr(C)]
pub struct ZrlRollout { pub rewards: *const f32, pub values: *const f32,
                        pub dones: *const u8, pub last_values: *const f32,
                        pub n_envs: i64, pub t: i64 }
#[repr(C)]
pub struct ZrlBatch { pub obs: *const f32, pub critic_obs: *const f32,
                      pub action: *const f32, pub mean_old: *const f32,
                      pub logp_old: *const f32, pub value_old: *const f32,
                      pub adv: *mut f32, pub ret: *const f32, pub n: i64,
                      pub n_global: i64, pub row_offset: i64,
                      pub on_device: i32, pub write_back_adv: i32 }

extern "C" {
    pub fn zrl_create(cfg: *const ZrlModelConfig, device: c_int,
                      comm: *const ZrlComm, out: *mut *mut ZrlCtx) -> c_int;
    pub fn zrl_destroy(ctx: *mut ZrlCtx) -> c_int;
    pub fn zrl_last_error(ctx: *const ZrlCtx) -> *const c_char;
    pub fn zrl_param_count(ctx: *const ZrlCtx) -> i64;
    pub fn zrl_init_reference(ctx: *mut ZrlCtx, init_noise_std: f32, init_lr: f32,
                              lcg_state: *mut u64) -> c_int;
    pub fn zrl_set_params(ctx: *mut ZrlCtx, flat: *const f32, count: i64) -> c_int;
    pub fn zrl_get_params(ctx: *mut ZrlCtx, flat: *mut f32, count: i64) -> c_int;
    pub fn zrl_set_normalizers(ctx: *mut ZrlCtx, om: *const f32, om2: *const f32, oc: f32,
                               cm: *const f32, cm2: *const f32, cc: f32) -> c_int;
    pub fn zrl_record_obs(ctx: *mut ZrlCtx, obs: *const f32, cobs: *const f32, n: i64) -> c_int;
    pub fn zrl_record_obs_ex(ctx: *mut ZrlCtx, obs: *const f32, cobs: *const f32, n: i64,
                             on_device: i32, mode: i32) -> c_int;
    // the frozen-normalizer flow: PendingNorm::push / Normalizer::commit
    pub fn zrl_pending_push(ctx: *mut ZrlCtx, obs: *const f32, cobs: *const f32, n: i64,
                            on_device: i32, mode: i32) -> c_int;
    pub fn zrl_commit_pending(ctx: *mut ZrlCtx) -> c_int;
    pub fn zrl_get_pending(ctx: *mut ZrlCtx, om: *mut f32, om2: *mut f32, oc: *mut f32,
                           cm: *mut f32, cm2: *mut f32, cc: *mut f32) -> c_int;
    pub fn zrl_set_lr(ctx: *mut ZrlCtx, lr: f32) -> c_int;
    pub fn zrl_get_lr(ctx: *mut ZrlCtx, lr: *mut f32) -> c_int;
    pub fn zrl_gae(ctx: *mut ZrlCtx, rewards: *const f32, values: *const f32,
                   dones: *const u8, last_values: *const f32, n_envs: i64, t: i64,
                   gamma: f32, lam: f32, adv: *mut f32, ret: *mut f32,
                   on_device: i32) -> c_int;
    pub fn zrl_update(ctx: *mut ZrlCtx, cfg: *const ZrlPpoConfig,
                      batch: *mut ZrlBatch, out: *mut ZrlStats) -> c_int;
    pub fn zrl_forward(ctx: *mut ZrlCtx, obs: *const f32, cobs: *const f32, n: i64,
                       mean: *mut f32, value: *mut f32, on_device: i32) -> c_int;
    pub fn zrl_policy_step(ctx: *mut ZrlCtx, obs: *const f32, cobs: *const f32, n: i64,
                           seed: u64, counter: u64, action: *mut f32, logp: *mut f32,
                           mean: *mut f32, value: *mut f32, on_device: i32) -> c_int;
    pub fn zrl_policy_step_lcg(ctx: *mut ZrlCtx, obs: *const f32, cobs: *const f32, n: i64,
                               lcg_state: *mut u64, action: *mut f32, logp: *mut f32,
                               mean: *mut f32, value: *mut f32, on_device: i32) -> c_int;
    pub fn zrl_save(ctx: *mut ZrlCtx, path: *const c_char) -> c_int;
    pub fn zrl_load(ctx: *mut ZrlCtx, path: *const c_char) -> c_int;
    pub fn zrl_load_from_bytes(ctx: *mut ZrlCtx, bytes: *const u8, len: usize) -> c_int;
    pub fn zrl_stream(ctx: *mut ZrlCtx) -> *mut c_void;
    pub fn zrl_synchronize(ctx: *mut ZrlCtx) -> c_int;
    pub fn zrl_abi_version() -> i32;
    pub fn zrl_nccl_unique_id(out: *mut u8) -> c_int;        // 128 bytes
    pub fn zrl_gae_update(ctx: *mut ZrlCtx, cfg: *const ZrlPpoConfig,
                          rollout: *const ZrlRollout, batch: *mut ZrlBatch,
                          out: *mut ZrlStats) -> c_int;
    pub fn zrl_gae_normalize_noalloc(rewards: *const f32, values: *const f32,
                                     dones: *const u8, last_values: *const f32,
                                     n_envs: i64, t: i64, gamma: f32, lam: f32,
                                     adv: *mut f32, ret: *mut f32, adv_norm: *mut f32,
                                     stream: *mut c_void) -> c_int;
    pub fn zrl_set_adam_state(ctx: *mut ZrlCtx, t3: *const i32, m: *const f32,
                              v: *const f32, count: i64) -> c_int;
    pub fn zrl_get_adam_state(ctx: *mut ZrlCtx, t3: *mut i32, m: *mut f32, v: *mut f32,
                              count: i64) -> c_int;
    pub fn zrl_get_normalizers(ctx: *mut ZrlCtx, om: *mut f32, om2: *mut f32, oc: *mut f32,
                               cm: *mut f32, cm2: *mut f32, cc: *mut f32) -> c_int;
    // parity hooks: the two halves of minibatch_step (ppo.rs:388-489)
    pub fn zrl_minibatch_grads(ctx: *mut ZrlCtx, cfg: *const ZrlPpoConfig,
                               batch: *const ZrlBatch, idx: *const i64, n_idx: i64,
                               grads: *mut f32, sums3: *mut f32) -> c_int;
    pub fn zrl_apply_grads(ctx: *mut ZrlCtx, cfg: *const ZrlPpoConfig, grads: *const f32,
                           kl: f32) -> c_int;
    pub fn zrl_gemm(ctx: *mut ZrlCtx, layout: i32, m: i32, n: i32, k: i32, a: *const f32,
                    lda: i32, b: *const f32, ldb: i32, c: *mut f32, ldc: i32,
                    split_k: i32) -> c_int;
    // Lcg and the epoch orders (rng.rs, ppo.rs:356-367)
    pub fn zrl_lcg_new(seed: u64) -> u64;
    pub fn zrl_lcg_unit(state: *mut u64) -> f32;
    pub fn zrl_lcg_gauss(state: *mut u64) -> f32;
    pub fn zrl_shuffle(seed: u64, n: i64, order: *mut i64);
    pub fn zrl_shuffle_device(ctx: *mut ZrlCtx, seed: u64, n: i64, order: *mut i32) -> c_int;
    pub fn zrl_rank_orders(seed: u64, n_global: i64, n_local: i64, row_offset: i64,
                           minibatches: i32, order: *mut i32, counts: *mut i64) -> i64;
    pub fn zrl_rank_orders_device(ctx: *mut ZrlCtx, seed: u64, n_global: i64, n_local: i64,
                                  row_offset: i64, minibatches: i32, order: *mut i32,
                                  counts: *mut i64) -> i64;
    pub fn zrl_set_mirror(ctx: *mut ZrlCtx, obs_perm: *const i32, obs_sign: *const f32,
                          cobs_perm: *const i32, cobs_sign: *const f32, act_perm: *const i32,
                          act_sign: *const f32) -> c_int;
    // failure handling
    pub fn zrl_set_wait_limit(ctx: *mut ZrlCtx, ns: u64) -> c_int;
    pub fn zrl_test_stall_next_gemm(ctx: *mut ZrlCtx) -> c_int;
    pub fn zrl_test_comm_wait(scenario: i32, timeout_ms: i32, aborted: *mut i32) -> c_int;
    // instrumentation
    pub fn zrl_kernel_launches(ctx: *const ZrlCtx) -> i64;
    pub fn zrl_set_profiling(ctx: *mut ZrlCtx, enabled: i32) -> c_int;
    pub fn zrl_get_profile(ctx: *mut ZrlCtx, gemm_ms: *mut f32, update_ms: *mut f32,
                           gemm_launches: *mut i64) -> c_int;
    pub fn zrl_profile_site(ctx: *const ZrlCtx, i: i32, name: *mut *const c_char,
                            ms: *mut f32, spans: *mut i64) -> i32;
}
