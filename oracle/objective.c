/*
 * Test infrastructure (not product code): a float64 CPU restatement of the reference's PPO
 * output-gradient kernel, ppo_output_gradient_kernel (src/ppo.cu:453-565), the same arithmetic
 * as oracle/ppo_ref.py's objective_gradient but in C so the GPU tests can check the objective
 * over a whole config-2 rollout (4.19 M samples x 256 slots) in seconds. Built by
 * oracle/Makefile into _ref/libt8oracle.so; pinned to ppo_ref.py by tests/test_ppo_oracle.py.
 *
 * t8or_objective(): for samples [0, n) of [n][k + 1] outputs (k logits, then the value) writes
 *   grads[n][k + 1] (float64) = d(mean objective over `batch` samples)/d(logits, value),
 *   margin[n]: 1 when the sample sits within `tolerance` of a branch of the objective that is
 *     discontinuous in its gradient (the policy ratio at 1 +- clip, or the value delta at
 *     +-value_clip, or the clipped and unclipped value losses equal outside the clip), where float32 and float64
 *     evaluations may legitimately take different branches;
 *   sums[8] += policy loss, value loss, entropy, KL, clip fraction, 0, decisions, decision entropy.
 * Samples are split over `threads` POSIX threads; sums are added per thread, then in thread order.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    const float* out;
    const uint8_t* masks;
    const int64_t* actions;
    const float *old_lp, *old_v, *adv, *ret;
    size_t begin, end;
    int k;
    double batch, clip, value_clip, value_coef, entropy_coef, tolerance;
    double* grads;
    uint8_t* margin;
    double sums[8];
} Job;

static void sample(Job* job, size_t i) {
    const int k = job->k;
    const float* o = job->out + i * (size_t)(k + 1);
    const uint8_t* m = job->masks + i * (size_t)k;
    double* g = job->grads + i * (size_t)(k + 1);
    int any = 0;
    for (int a = 0; a < k; ++a) any |= m[a] != 0;
    /* the legal set: the mask, or action 0 alone when nothing is legal (src/ppo.cu:476-489) */
#define LEGAL(a) (any ? m[(a)] != 0 : (a) == 0)
    double maximum = -INFINITY;
    for (int a = 0; a < k; ++a) {
        if (LEGAL(a) && o[a] > maximum) maximum = o[a];
    }
    double total = 0.0;
    for (int a = 0; a < k; ++a) {
        if (LEGAL(a)) total += exp((double)o[a] - maximum);
    }
    if (total < 1e-20) total = 1e-20;
    const double log_sum = log(total) + maximum;
    const int selected = any ? (int)job->actions[i] : 0;
    const double log_ratio = ((double)o[selected] - log_sum) - job->old_lp[i];
    const double ratio = exp(log_ratio);
    const double advantage = job->adv[i];
    const double unclipped = ratio * advantage;
    double clipped_ratio = ratio;
    if (clipped_ratio > 1.0 + job->clip) clipped_ratio = 1.0 + job->clip;
    if (clipped_ratio < 1.0 - job->clip) clipped_ratio = 1.0 - job->clip;
    const double clipped = clipped_ratio * advantage;
    const int use_unclipped = unclipped <= clipped;
    const double policy_loss = -(unclipped < clipped ? unclipped : clipped);
    const double lp_grad = use_unclipped ? -advantage * ratio : 0.0;
    double entropy = 0.0;
    int legal_count = 0;
    for (int a = 0; a < k; ++a) {
        if (!LEGAL(a)) continue;
        const double lp = (double)o[a] - log_sum;
        entropy -= exp(lp) * lp;
        ++legal_count;
    }
    for (int a = 0; a < k; ++a) {
        if (!LEGAL(a)) {
            g[a] = 0.0;
            continue;
        }
        const double lp = (double)o[a] - log_sum;
        const double p = exp(lp);
        g[a] = (lp_grad * ((a == selected ? 1.0 : 0.0) - p)) / job->batch +
               job->entropy_coef * p * (lp + entropy) / job->batch;
    }
#undef LEGAL
    const double value = o[k];
    const double error = value - job->ret[i];
    double value_gradient = error;
    double value_loss = 0.5 * error * error;
    int near = fabs(ratio - (1.0 + job->clip)) <= job->tolerance || fabs(ratio - (1.0 - job->clip)) <= job->tolerance;
    if (job->value_clip > 0.0) {
        const double delta = value - job->old_v[i];
        double bounded = delta;
        if (bounded > job->value_clip) bounded = job->value_clip;
        if (bounded < -job->value_clip) bounded = -job->value_clip;
        const double clipped_error = (job->old_v[i] + bounded) - job->ret[i];
        const double clipped_loss = 0.5 * clipped_error * clipped_error;
        if (clipped_loss > value_loss) {
            value_loss = clipped_loss;
            value_gradient = fabs(delta) <= job->value_clip ? clipped_error : 0.0;
        }
        /* inside the clip the two losses are equal and either branch gives the same gradient;
           outside it the clipped branch has none, so the losses' crossing is a switch */
        near = near || fabs(fabs(delta) - job->value_clip) <= job->tolerance ||
               (fabs(delta) > job->value_clip &&
                fabs(clipped_loss - 0.5 * error * error) <= job->tolerance * (clipped_loss + 1e-30));
    }
    g[k] = job->value_coef * value_gradient / job->batch;
    if (job->margin) job->margin[i] = (uint8_t)near;
    job->sums[0] += policy_loss;
    job->sums[1] += value_loss;
    job->sums[2] += entropy;
    job->sums[3] += (ratio - 1.0) - log_ratio;
    job->sums[4] += fabs(ratio - 1.0) > job->clip ? 1.0 : 0.0;
    if (legal_count > 1) {
        job->sums[6] += 1.0;
        job->sums[7] += entropy;
    }
}

static void* run(void* arg) {
    Job* job = (Job*)arg;
    for (size_t i = job->begin; i < job->end; ++i) sample(job, i);
    return NULL;
}

int t8or_objective(const float* out, const uint8_t* masks, const int64_t* actions, const float* old_lp,
                   const float* old_v, const float* adv, const float* ret, size_t n, int k, double batch, float clip,
                   float value_clip, float value_coef, float entropy_coef, double tolerance, double* grads,
                   uint8_t* margin, double* sums, int threads) {
    if (threads < 1) threads = 1;
    if ((size_t)threads > n) threads = n > 0 ? (int)n : 1;
    Job* jobs = calloc((size_t)threads, sizeof(Job));
    pthread_t* ids = calloc((size_t)threads, sizeof(pthread_t));
    if (!jobs || !ids) {
        free(jobs);
        free(ids);
        return 1;
    }
    for (int t = 0; t < threads; ++t) {
        Job* job = &jobs[t];
        job->out = out;
        job->masks = masks;
        job->actions = actions;
        job->old_lp = old_lp;
        job->old_v = old_v;
        job->adv = adv;
        job->ret = ret;
        job->begin = n * (size_t)t / (size_t)threads;
        job->end = n * (size_t)(t + 1) / (size_t)threads;
        job->k = k;
        job->batch = batch;
        job->clip = clip;
        job->value_clip = value_clip;
        job->value_coef = value_coef;
        job->entropy_coef = entropy_coef;
        job->tolerance = tolerance;
        job->grads = grads;
        job->margin = margin;
        if (t > 0) pthread_create(&ids[t], NULL, run, job);
    }
    run(&jobs[0]);
    for (int t = 1; t < threads; ++t) pthread_join(ids[t], NULL);
    for (int t = 0; t < threads; ++t) {
        for (int s = 0; s < 8; ++s) sums[s] += jobs[t].sums[s];
    }
    free(jobs);
    free(ids);
    return 0;
}
