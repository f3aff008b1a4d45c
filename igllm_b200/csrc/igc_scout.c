/* igc_scout.c - the n-gram proposer, host C.
 *
 * The reference's scout (app_core.c:12277-12361): a growing list of the ids a
 * stream has committed and a backward scan for the latest earlier place the
 * last `reach` ids appeared, longest reach (3) first, then 2.  It is a few
 * hundred thousand integer compares at most, sequential by nature, and stays
 * on the host beside the round loop that feeds it.
 */
#include <stdlib.h>
#include <string.h>

#include "../../include/igllm_cuda.h"

#define SCOUT_REACH 3       /* app_core.c:12270 */
#define SCOUT_REACH_LEAST 2 /* app_core.c:12271 */

struct igc_scout {
  int32_t *ids;
  int count;
  int room;
};

int igc_scout_open(igc_scout **scout_out) {
  if (!scout_out) return IGC_FAIL_ARGUMENT;
  *scout_out = (igc_scout *)calloc(1, sizeof(igc_scout));
  return *scout_out ? IGC_OKAY : IGC_FAIL_MEMORY;
}

void igc_scout_close(igc_scout *scout) {
  if (!scout) return;
  free(scout->ids);
  free(scout);
}

void igc_scout_clear(igc_scout *scout) {
  if (scout) scout->count = 0;
}

int igc_scout_span(const igc_scout *scout) { return scout ? scout->count : 0; }

/* Only ids the model agreed to are noted, so the scout never learns from its
 * own rejected guesses. */
int igc_scout_note(igc_scout *scout, const int32_t *id_list, int id_count) {
  if (!scout || id_count < 0 || (!id_list && id_count > 0)) return IGC_FAIL_ARGUMENT;
  if (id_count == 0) return IGC_OKAY;
  if (scout->count + id_count > scout->room) {
    int want = scout->room ? scout->room : 1024;
    int32_t *grown;
    while (want < scout->count + id_count) want *= 2;
    grown = (int32_t *)realloc(scout->ids, sizeof(int32_t) * (size_t)want);
    if (!grown) return IGC_FAIL_MEMORY;
    scout->ids = grown;
    scout->room = want;
  }
  memcpy(scout->ids + scout->count, id_list, sizeof(int32_t) * (size_t)id_count);
  scout->count += id_count;
  return IGC_OKAY;
}

int igc_scout_draw(const igc_scout *scout, int32_t *id_out, int want_count) {
  if (!scout || !id_out || want_count < 1) return 0;
  for (int reach = SCOUT_REACH; reach >= SCOUT_REACH_LEAST; --reach) {
    const int32_t *tail;
    if (scout->count < reach + 1) continue;
    tail = scout->ids + scout->count - reach;
    for (int place = scout->count - reach - 1; place >= 0; --place) {
      int slot = 0, take;
      while (slot < reach && scout->ids[place + slot] == tail[slot]) ++slot;
      if (slot < reach) continue;
      take = scout->count - (place + reach);
      if (take < 1) continue;
      if (take > want_count) take = want_count;
      memcpy(id_out, scout->ids + place + reach, sizeof(int32_t) * (size_t)take);
      return take;
    }
  }
  return 0;
}
