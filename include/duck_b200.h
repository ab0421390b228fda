/* duck_gym_b200 -- C ABI of the B200 AVBD environment-step library.
 *
 * This is the drop-in boundary for the reference's CUDA entry points: the
 * pybind11 class `_duck_cuda.CudaBatch` defined in src/cuda/extension.cu
 * (Interface at :160-173, Batch<S> at :187-422, makeBatch at :423-435, module
 * at :436-452).  The reference binds those methods to torch tensors; here every
 * entry point takes plain device pointers, element counts and a cudaStream_t,
 * so any host language can bind it (the Python binding lives in
 * duck_gym_b200/cuda_batch.py and reproduces the reference's Python API).
 *
 * Conventions (same as the reference's Batch, extension.cu:203-213):
 *  - A batch lives on one device.  Every call runs asynchronously on the
 *    given stream; calls are serialised across streams by a private event
 *    (the reference's wait()/record()).  Only duck_batch_create and
 *    duck_batch_destroy synchronise.
 *  - Real is float for fp64 == 0 and double for fp64 == 1.  Arrays are dense,
 *    C-contiguous, on the batch's device, with the shapes given below
 *    (E envs, B bodies, J joints).
 *  - Numeric failures never raise: they set the sticky per-env flag exported
 *    as diag[:, 5], which reset clears (kernel.cuh:382).
 *  - Argument errors return a nonzero status; duck_last_error() describes
 *    the most recent one on the calling thread.
 */
#ifndef DUCK_B200_H
#define DUCK_B200_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct duck_batch duck_batch;
typedef struct CUstream_st *duck_stream; /* == cudaStream_t */

enum { DUCK_OK = 0, DUCK_EINVAL = 1, DUCK_ECUDA = 2, DUCK_EMODEL = 3 };

/* Message of the last failed call on this thread ("" if none). */
const char *duck_last_error(void);

/* Replaces CudaBatch.__init__ / makeBatch (extension.cu:216-265, 423-435).
 * Loads a DUCK_MODEL v1/v2 file (solver.cpp:67-174), converts it
 * (model.hpp:237-360) and initialises num_envs environments.
 * Requires 0 < num_envs <= 65536, dt > 0 finite, iterations > 0.
 * specialized requires the 16-body / 14-hinge MicroDuck joint layout
 * (extension.cu:225-237); shared_memory requires specialized.  Both flags
 * are accepted for API compatibility: this library always keeps each
 * environment's working state on chip, so they select no other code path. */
int duck_batch_create(const char *model_path, int num_envs, double dt, int iterations, int device,
                      int fp64, int specialized, int shared_memory, duck_stream stream,
                      duck_batch **out);
/* Options of duck_batch_create_ex (extensions beyond the reference). */
typedef struct duck_batch_options {
  /* Largest accepted number of body-collision pairs.  32 is the reference's
   * limit (solver.cpp:151-152, model.hpp:26-29) and what duck_batch_create
   * uses; up to 128 accepts models the reference rejects (for example all 91
   * non-adjacent link pairs of the 15-link biped).  The contact bound
   * (pairs + 4 per ground shape <= 160) still applies. */
  int max_pairs;
} duck_batch_options;

/* duck_batch_create with options (NULL = the reference's limits). */
int duck_batch_create_ex(const char *model_path, int num_envs, double dt, int iterations, int device,
                         int fp64, int specialized, int shared_memory, const duck_batch_options *options,
                         duck_stream stream, duck_batch **out);

/* Replaces Batch::~Batch (extension.cu:266-272). */
void duck_batch_destroy(duck_batch *batch);

/* Sizes: out[0] E, out[1] B, out[2] J, out[3] contact bound, out[4] portable
 * record length (Reals), out[5] fp64, out[6] device, out[7] environments per
 * CTA, out[8] lanes per environment, out[9] shared bytes per CTA. */
int duck_batch_info(const duck_batch *batch, int32_t *out);
/* No reference counterpart.  Model sizes: out[0] bodies, out[1] joints,
 * out[2] collision shapes, out[3] body-collision pairs. */
int duck_batch_model_counts(const duck_batch *batch, int32_t *out);
/* Joint name i (the reference's joint_names property, extension.cu:416-421). */
const char *duck_batch_joint_name(const duck_batch *batch, int index);

/* Replaces Batch::reset (extension.cu:273-284, kernel resetStates :29-50).
 * mask [E] uint8 (bool), q [E,J], roots [E,6] (xyz + rotation vector). */
int duck_batch_reset(duck_batch *batch, const uint8_t *mask, const void *q, const void *roots,
                     duck_stream stream);

/* Replaces Batch::step (extension.cu:285-306, kernel advance :78-114):
 * implicit PD targets [E,J], base forces [E,3], substeps > 0, kp >= 0,
 * limit >= 0 (0 = uncapped). */
int duck_batch_step(duck_batch *batch, const void *target, const void *forces, int substeps,
                    double kp, double limit, duck_stream stream);

/* Replaces Batch::stepMotor (extension.cu:307-320, kernel advanceMotor
 * :115-127): motor [E,J,3] = (torque, dry-friction budget, viscous damping)
 * held for one physics step, base forces [E,3]. */
int duck_batch_step_motor(duck_batch *batch, const void *motor, const void *forces,
                          duck_stream stream);

/* Replaces Batch::state (extension.cu:321-335, kernel snapshot :128-138):
 * bodies [E,B,13] (x, q wxyz, v, w), joints [E,J,2] (angle, rate),
 * diag [E,6] (joint error, penetration, contacts, converged, axis error,
 * failed). */
int duck_batch_state(duck_batch *batch, void *bodies, void *joints, void *diag,
                     duck_stream stream);

/* Replaces Batch::contactForces (extension.cu:336-347): [E,B,3]. */
int duck_batch_contact_forces(duck_batch *batch, void *out, int ground_only, duck_stream stream);
/* Replaces Batch::selfContactStats (extension.cu:348-359): [E,2]. */
int duck_batch_self_contact_stats(duck_batch *batch, void *out, duck_stream stream);
/* Replaces Batch::contactCounts (extension.cu:360-370): [E,2]. */
int duck_batch_contact_counts(duck_batch *batch, void *out, duck_stream stream);
/* Replaces Batch::generalizedLoads (extension.cu:371-384): offset [E,3],
 * out [E,J,3] = (bias, contact+limit, applied actuator) per hinge. */
int duck_batch_generalized_loads(duck_batch *batch, const void *offset, void *out,
                                 duck_stream stream);

/* Replaces Batch::reference (extension.cu:385-415): one environment of the
 * same model advanced from its initial state on the HOST, for quick checks.
 * target [J], forces [3], outputs bodies [B,13], joints [J,2], diag [6], all
 * host pointers.  Unlike the reference (which re-runs its solver on the CPU),
 * this runs the device kernel on a scratch single-env batch and copies back. */
int duck_batch_reference(duck_batch *batch, const void *target, const void *forces, int substeps,
                         double kp, double limit, void *bodies, void *joints, void *diag);

/* No counterpart in the reference: an allocation-free duck_batch_reference.
 * Same arguments, same results (per-environment parameters included: the one
 * environment uses environment 0's values, as duck_batch_reference does).
 * duck_batch_reference takes its scratch (a one-environment state record plus
 * staging for inputs and outputs) from cudaMalloc; this entry point calls no
 * cudaMalloc, cudaFree or allocating library routine.  It is for callers that
 * cannot allocate device memory when they want this check: a host framework
 * whose caching allocator owns the device memory and forbids raw cudaMalloc
 * beside it, a process held to a fixed device-memory budget, and real-time
 * control loops that must not take the implicit synchronisation of
 * cudaMalloc/cudaFree.  It gives no allocation and nothing more: like
 * duck_batch_reference it is synchronous, copies from and to host memory with
 * cudaMemcpy and runs on the legacy default stream.
 * Its scratch is a file-scope device array of 32 KiB that every GPU loading
 * the library holds until exit; models whose record and staging need more are
 * rejected with DUCK_EINVAL and a message giving both sizes (the seed biped
 * needs 10 KiB in fp32, 20 KiB in fp64).  The first call on a device resolves
 * the array's device address with that device current and caches it for the
 * process; after a cudaDeviceReset of the device the cached address is stale,
 * so do not use this entry point on a device after resetting it.  All calls
 * share the array and it keeps the previous call's contents (each call clears
 * the record before use), so calls that overlap on the GPU race: serialise
 * them.  Inputs and outputs are host pointers, as for duck_batch_reference. */
int duck_batch_reference_static(duck_batch *batch, const void *target, const void *forces,
                                int substeps, double kp, double limit, void *bodies, void *joints,
                                void *diag);

/* No reference counterpart.  Copies environments [first, first + count) to
 * or from a dense array of portable records ([count, record length] Reals,
 * device memory); the layout is the one written by oracle/avbd_oracle.cpp:
 * header 8, bodies B x 16, joints J x 22, contacts bound x 32.  Used to load
 * one state into both this library and the CPU oracle, and for checkpoints. */
int duck_batch_export(duck_batch *batch, int first, int count, void *records, duck_stream stream);
int duck_batch_import(duck_batch *batch, int first, int count, const void *records,
                      duck_stream stream);

/* No reference counterpart.  Contact keys of one environment copied to the
 * host: keys [capacity,5] int32 rows (body, shape, feature, other,
 * otherShape); returns the contact count through *count. */
int duck_batch_contact_keys(duck_batch *batch, int env, int32_t *keys, int capacity, int *count,
                            duck_stream stream);

/* Tensor environment (the reference's python/duck_gym/tensor_env.py step math)
 * fused into three kernels that read the batch's physics state directly.
 * Buffers are device arrays of the batch dtype (Real) unless noted; episode
 * lengths are int64, returns, observations and rewards float32, masks bool.
 * task: 0 standing, 1 locomotion; filter: velocity filter on (locomotion);
 * tilt: -cos(0.5) as the env computes it on its device. */
typedef struct duck_env_params {
  int task, filter, max_episode_length;
  double root_height, tilt, control_dt, velocity_alpha, tracking_weight, heading_weight, tracking_sigma,
      gait_period;
  double iquat[4]; /* conjugated root principal-frame quaternion (w, x, y, z) */
  /* Gait shaping from the env's gait.npz (tensor_env.py:152-171): the gait
   * reference targets (gait), the foot-clearance and load-transfer rewards.
   * gait_table [4 directions, gait_samples, J] and foot_xyz [2, foot_points, 3]
   * (foot collision points in foot-body coordinates) are Real device arrays;
   * mass is the robot's total mass. */
  int gait, foot_clearance, load_transfer, gait_samples, foot_points;
  int foot_body[2];
  double gait_lift, mass;
  const void *gait_table, *foot_xyz;
} duck_env_params;

/* Observation width of the environment described by params (52, 58 or 60 for
 * the 14-joint biped). */
int duck_env_obs_dim(const duck_batch *batch, const duck_env_params *params);

/* tensor_env.py:280-283: a = clamp(actions, -1, 1), target = clamp(home +
 * scale a, lower, upper).  actions, a_out, target_out [E,J]; home, lower,
 * upper [J]. */
int duck_env_targets(duck_batch *batch, const void *actions, double scale, const void *home,
                     const void *lower, const void *upper, void *a_out, void *target_out,
                     duck_stream stream);

/* tensor_env.py:263-283: a = clamp(actions, -1, 1), target = clamp(ref + scale a,
 * lower, upper) where ref is HOME or, with params->gait, the gait table at the
 * episode phase in the command's direction blended in over the first second.
 * episode_length [E] int64 and commands [E,2] are the env buffers before the
 * step. */
int duck_env_reference_targets(duck_batch *batch, const duck_env_params *params, const void *actions,
                               double scale, const void *home, const void *lower, const void *upper,
                               const int64_t *episode_length, const void *commands, void *a_out,
                               void *target_out, duck_stream stream);

/* tensor_env.py:291-361 after the physics step: projected gravity and body
 * velocities, termination (failed), reward, time-outs, done, episode
 * lengths (+1), returns (+reward), prev_actions := a, velocity filter, and the
 * terminal observation obs [E,D].  Optional outputs (NULL to skip): diag
 * [E,6] as duck_batch_state writes it, and tracking [E,4] float32 with the
 * per-env terms of the locomotion log (|v_xy - command|, v_xy . command,
 * sqrt of the reward's velocity error, |heading angle|). */
int duck_env_post_step(duck_batch *batch, const duck_env_params *params, const void *home,
                       const void *a, void *prev_actions, int64_t *episode_length, float *returns,
                       const void *commands, void *filtered, float *obs, float *reward,
                       uint8_t *failed, uint8_t *timeout, uint8_t *done, void *diag, float *tracking,
                       duck_stream stream);

/* tensor_env.py:238-261: observations [E,D] of the current state. */
int duck_env_observe(duck_batch *batch, const duck_env_params *params, const void *home,
                     const void *actions, const int64_t *episode_length, const void *commands,
                     const void *filtered, float *obs, duck_stream stream);

/* tensor_env.py:197-219: for masked environments zero prev_actions [E,J],
 * forces [E,3], episode_length, returns and filtered [E,2], and copy
 * new_commands [E,2] into commands (new_commands may be NULL). */
int duck_env_reset_buffers(duck_batch *batch, const uint8_t *mask, void *prev_actions, void *forces,
                           int64_t *episode_length, float *returns, void *filtered, void *commands,
                           const void *new_commands, duck_stream stream);

/* BAM environment (the reference's python/duck_gym/bam_env.py with the
 * XL330/m6 servo of actuator.py:16-77 and the walking reward of
 * walking_reward.py) fused into kernels that read the batch's physics state
 * directly.  Settings come from the env's config.json and training dictionary
 * (bam_env.py:33-133).  J <= 32, two feet. */
typedef struct duck_bam_params {
  int lag, decimation, max_episode_length, source_iteration;
  int neutral_head, heading_hold, reward_enabled;
  int head_stability, mean_velocity, heading_reward; /* optional terms (bam_env.py:358-381) */
  int foot_body[2];
  uint32_t head_mask;     /* bit j: joint j is a head or neck joint */
  uint32_t override_mask; /* bit t: walking weight t replaced by overrides[t] */
  double dt, step_dt;     /* physics and control step */
  double kp_fw, vin, vin_drop_gain, vin_min, force_limit;
  double kt, R, friction_base, friction_stribeck, load_friction_external, load_friction_motor,
      load_friction_external_stribeck, load_friction_motor_stribeck, load_friction_external_quad,
      load_friction_motor_quad, dtheta_stribeck, alpha, friction_viscous;
  double root_iquat[4];   /* conjugated root principal-frame quaternion */
  double foot_site[2][3]; /* sole sites in foot-body coordinates */
  double linear_variance, vertical_variance, mean_velocity_alpha, mean_velocity_variance,
      mean_velocity_weight, heading_reward_weight, heading_reward_variance, head_position_weight,
      head_velocity_weight;
  double tilt_limit;      /* -cos(70 deg) */
  double overrides[15];   /* walking weights in walking_reward.py:108-122 order */
  double stand_std[32], walk_std[32], soft_limits[32][2];
} duck_bam_params;

/* Device buffers of one BAM environment batch ([E,...], Real unless noted).
 * Names follow the reference BamEnv attributes. */
typedef struct duck_bam_buffers {
  const void *home, *root_offset, *zero_forces;     /* [E,J], [E,3], [E,3] zeros */
  void *action, *old_action, *previous_motor, *previous_applied, *observed_velocity; /* [E,J] */
  void *command, *mean_velocity_world;             /* [E,3] */
  void *target_yaw, *self_contacts, *self_penetration; /* [E] */
  void *air_time, *contact_time, *peak_height;     /* [E,2] */
  void *contact_force;                             /* [E,2,3] */
  void *joints;                                    /* [E,J,2] */
  void *head_ema;                                  /* [E,4] */
  void *target_history;                            /* [lag+1,E,J] */
  void *motor;                                     /* [E,J,3] scratch: motor channels */
  void *features;                                  /* [E,29]: root quat, gravity, ang_vel, lin_vel,
                                                      root-origin world velocity, site pos [2,3],
                                                      site vel [2,3], numeric-failure flag */
  void *terms;                                     /* [E,19] reward terms */
  uint8_t *contact, *history_initialized;          /* bool [E,2], [E] */
  uint8_t *done, *timeout, *failed;                /* bool [E] */
  int64_t *episode_length;                         /* [E] */
  int32_t *counters;                               /* [2]: delay-ring cursor, common step counter */
  float *obs_actor, *obs_critic, *reward;          /* [E,19+3J], [E,duck_bam_critic_dim], [E] */
  void *servo_supply;                              /* [E] scratch: servo supply voltage */
} duck_bam_buffers;

/* Critic observation width (76 for 14 joints, +3 with the mean-velocity
 * filter, +1 with the heading reward). */
int duck_bam_critic_dim(const duck_batch *batch, const duck_bam_params *params);
/* bam_env.py:292-389: one control step -- prologue, decimation x (servo,
 * one physics substep, bookkeeping), reward, masks and observations.
 * actions [E,J] Real.  Launches only kernels (no host synchronisation), so
 * the sequence can be captured into a CUDA graph. */
int duck_bam_step(duck_batch *batch, const duck_bam_params *params, const duck_bam_buffers *buffers,
                  const void *actions, duck_stream stream);
/* The parts of duck_bam_step, for per-substep callbacks:
 * begin (:292-303), one substep (:305-344), finish (:345-389). */
int duck_bam_begin(duck_batch *batch, const duck_bam_params *params, const duck_bam_buffers *buffers,
                   const void *actions, duck_stream stream);
int duck_bam_substep(duck_batch *batch, const duck_bam_params *params, const duck_bam_buffers *buffers,
                     duck_stream stream);
int duck_bam_finish(duck_batch *batch, const duck_bam_params *params, const duck_bam_buffers *buffers,
                    duck_stream stream);
/* The servo alone (delay ring, generalized loads, XL330/m6) writing the motor
 * channels of one substep without stepping the physics. */
int duck_bam_servo(duck_batch *batch, const duck_bam_params *params, const duck_bam_buffers *buffers,
                   duck_stream stream);
/* bam_env.py:245-275: zero the buffers of the masked environments and refill
 * their delay ring with HOME (the physics reset is duck_batch_reset). */
int duck_bam_reset_buffers(duck_batch *batch, const duck_bam_params *params,
                           const duck_bam_buffers *buffers, const uint8_t *mask, duck_stream stream);
/* bam_env.py:136-211: refresh frames (features, joints, foot contacts) and
 * observations from the current physics state.  With update_heading set (the
 * end of reset, :270-275) the masked environments (mask may be NULL) first
 * take their current heading as target and the heading command is updated
 * when heading hold is on. */
int duck_bam_observe(duck_batch *batch, const duck_bam_params *params, const duck_bam_buffers *buffers,
                     const uint8_t *mask, int update_heading, duck_stream stream);

/* No reference counterpart (the reference shares one model across every
 * environment, kernel.cuh:331): per-environment physical parameters for
 * domain randomisation.  mass [E,B] body masses, inertia [E,B,3] principal
 * inertias, friction [E,S] ground friction of each collision shape -- device
 * arrays of Real, copied into the batch; NULL restores the model's values for
 * that quantity.  Static bodies (model mass 0) stay static.  Values take effect
 * from the next step: physics, generalized loads and the BAM servo use them.
 * A non-finite or non-positive mass or inertia of a dynamic body, or a
 * negative or non-finite friction, sets that environment's failure flag
 * (diag[:, 5]).  Body-pair friction keeps the model's values. */
int duck_batch_set_parameters(duck_batch *batch, const void *mass, const void *inertia,
                              const void *friction, duck_stream stream);

/* No reference counterpart.  Number of kernel launches issued by this batch
 * since creation (for launch accounting in benchmarks). */
int64_t duck_batch_launches(const duck_batch *batch);

/* No reference counterpart in this repository: the loss of rsl-rl's PPO
 * (third-party; the reference trains with it, scripts/train_bam_native.py:
 * 14-140) for one minibatch, fused with its gradient.  Inputs are device
 * float32 arrays: policy means mu [B,A], std [A], values [B], stored actions
 * [B,A], old log-probabilities [B], old means and stds [B,A], rollout values,
 * returns and normalised advantages [B].  Writes out[5] = (surrogate, value
 * loss, entropy, kl, loss) and the loss gradient with respect to mu [B,A],
 * std [A] and the values [B].  scratch holds duck_ppo_loss_scratch(B, A)
 * floats.  Two kernel launches on `stream`, no allocation, no host sync: it
 * can be captured in a CUDA graph.  A <= 32. */
int duck_ppo_loss_scratch(int batch, int actions);
int duck_ppo_loss(int batch, int actions, const float *mu, const float *std, const float *value, const float *act,
                  const float *old_log_prob, const float *old_mu, const float *old_sigma, const float *target_value,
                  const float *returns, const float *advantage, double clip, double value_coef,
                  double entropy_coef, float *scratch, float *out, float *grad_mu, float *grad_std,
                  float *grad_value, duck_stream stream);

/* No reference counterpart.  FP32 fused-multiply-add throughput probe used
 * as the roofline denominator: runs `iterations` dependent FMA chains on
 * every SM and returns achieved TFLOP/s (2 flops per FMA) in *tflops. */
int duck_fp32_peak(int device, int iterations, double *tflops, duck_stream stream);

#ifdef __cplusplus
}
#endif
#endif
