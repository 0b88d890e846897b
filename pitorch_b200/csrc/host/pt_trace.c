/*
 * pt_trace.c -- host span tracing with the API of pitorch/profiler/trace.c.
 * Chrome-trace JSON ("X" complete events, microsecond timestamps) as the
 * reference writes it (trace.c:89-120).
 */
#include <stdio.h>
#include <string.h>
#include <time.h>

#include "../../../include/trace.h"

uint32_t pt_time_us(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (uint32_t)((uint64_t)ts.tv_sec * 1000000u + (uint64_t)ts.tv_nsec / 1000u);
}

void pt_trace_init(pt_trace_t *t) {
    if (!t) return;
    memset(t, 0, sizeof(*t));
    t->enabled = 1;
}

void pt_trace_begin(pt_trace_t *t, const char *name, const char *cat, int layer) {
    if (!t || !t->enabled || t->depth >= PT_TRACE_MAX_DEPTH) return;
    int d = t->depth++;
    t->stack[d].name = name;
    t->stack[d].cat = cat;
    t->stack[d].ts_us = pt_time_us();
    t->stack[d].layer = (int8_t)layer;
}

void pt_trace_end(pt_trace_t *t) {
    if (!t || !t->enabled || t->depth <= 0) return;
    int d = --t->depth;
    uint32_t now = pt_time_us();
    if (t->count >= PT_TRACE_MAX_EVENTS) return;
    pt_trace_event_t *e = &t->events[t->count++];
    e->name = t->stack[d].name;
    e->cat = t->stack[d].cat;
    e->ts_us = t->stack[d].ts_us;
    e->dur_us = now - e->ts_us;
    e->layer = t->stack[d].layer;
    e->depth = (int8_t)d;
    e->hw_cycles = 0;
    e->hw_stall = 0;
}

void pt_trace_reset(pt_trace_t *t) {
    if (!t) return;
    t->count = 0;
    t->depth = 0;
}

void pt_trace_write_json(const pt_trace_t *t, const char *path) {
    if (!t) return;
    FILE *f = fopen(path, "w");
    if (!f) return;
    uint32_t t0 = t->count ? t->events[0].ts_us : 0;
    for (int i = 0; i < t->count; i++)
        if (t->events[i].ts_us < t0) t0 = t->events[i].ts_us;
    fprintf(f, "[\n");
    for (int i = 0; i < t->count; i++) {
        const pt_trace_event_t *e = &t->events[i];
        fprintf(f, "  {\"name\":\"%s\",\"cat\":\"%s\",\"ph\":\"X\",\"ts\":%u,\"dur\":%u,"
                   "\"pid\":0,\"tid\":0,\"args\":{\"layer\":%d,\"depth\":%d}}%s\n",
                e->name ? e->name : "?", e->cat ? e->cat : "", e->ts_us - t0, e->dur_us, e->layer,
                e->depth, i + 1 < t->count ? "," : "");
    }
    fprintf(f, "]\n");
    fclose(f);
}

void pt_trace_write_meta(const char *path, const char *name, const char *model, int dim, int layers,
                         int vocab, const char *device, int num_qpus, int steps, float lr,
                         float final_loss, float total_time_s, const char *notes) {
    FILE *f = fopen(path, "w");
    if (!f) return;
    fprintf(f, "{\"name\":\"%s\",\"model\":\"%s\",\"dim\":%d,\"layers\":%d,\"vocab\":%d,"
               "\"device\":\"%s\",\"num_qpus\":%d,\"steps\":%d,\"lr\":%g,\"final_loss\":%g,"
               "\"total_time_s\":%g,\"notes\":\"%s\"}\n",
            name ? name : "", model ? model : "", dim, layers, vocab, device ? device : "", num_qpus,
            steps, lr, final_loss, total_time_s, notes ? notes : "");
    fclose(f);
}
