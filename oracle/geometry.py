"""Station geometry oracle (float64 numpy), restating the reference's bias construction.

Reference: fore_swe/extended_dl_forecasting.py
  * pairwise_vector_angle            :20-30   Kahan's theta = 2*atan2(|| |u|v - |v|u ||, || |u|v + |v|u ||)
  * DataLoader.getHaversineDistance  :305-318 sklearn haversine_distances(deg2rad[lat, lon]) * 6371
  * DataLoader.getAlgularityOfLocations :320-344 per-station vector (R_km + elev_ft*0.3048) *
        (cos(lat)cos(lon), cos(lat)sin(lon), <x again>) -- the third component repeats x (z is computed
        and discarded, :333) and metres are added to a radius in km (:323-331); result in degrees (:339)
  * DataLoader.getDistanceAndAngularity :346-352 returns (distance_km, angle_deg), both [N, N] float64

The haversine itself is sklearn's (scikit-learn, pinned 1.3.2 in requirement_files/foreswe_requirement.txt:49;
1.9.0 here). Its published formula: d = 2*arcsin(sqrt(sin^2(dlat/2) + cos(lat1)cos(lat2)sin^2(dlon/2))).

TEST INFRASTRUCTURE: used by tests and the CPU baseline only.
"""
import numpy as np

EARTH_RADIUS_KM = 6371.0      # extended_dl_forecasting.py:314, :324
FEET_TO_METRES = 0.3048       # extended_dl_forecasting.py:323


def haversine_km(lat_deg, lon_deg):
    """[N] latitude, longitude in degrees -> [N, N] great-circle distance in km (float64)."""
    lat = np.deg2rad(np.asarray(lat_deg, dtype=np.float64))
    lon = np.deg2rad(np.asarray(lon_deg, dtype=np.float64))
    s_lat = np.sin(0.5 * (lat[:, None] - lat[None, :]))
    s_lon = np.sin(0.5 * (lon[:, None] - lon[None, :]))
    cos_lat = np.cos(lat)
    h = s_lat * s_lat + cos_lat[:, None] * cos_lat[None, :] * s_lon * s_lon
    return 2.0 * np.arcsin(np.sqrt(h)) * EARTH_RADIUS_KM


def station_vectors(lat_deg, lon_deg, elev_ft):
    """Per-station Cartesian vectors exactly as the reference builds them: [x, y, x] (see module doc)."""
    lat = np.asarray(lat_deg, dtype=np.float64)
    lon = np.asarray(lon_deg, dtype=np.float64)
    el = np.asarray(elev_ft, dtype=np.float64)
    radius = EARTH_RADIUS_KM + el * FEET_TO_METRES
    x = radius * np.cos(np.deg2rad(lat)) * np.cos(np.deg2rad(lon))
    y = radius * np.cos(np.deg2rad(lat)) * np.sin(np.deg2rad(lon))
    return np.stack([x, y, x], axis=1)


def pairwise_vector_angle(vectors):
    """[N, 3] -> [N, N] angle in radians by Kahan's formula (robust near 0 and pi)."""
    v = np.asarray(vectors, dtype=np.float64)
    n = np.sqrt(np.add.reduce(v * v, axis=1))
    a = n[:, None, None] * v[None, :, :]          # |u| v  with u = row i, v = row j
    b = n[None, :, None] * v[:, None, :]          # |v| u
    diff = np.sqrt(np.add.reduce((a - b) * (a - b), axis=2))
    summ = np.sqrt(np.add.reduce((a + b) * (a + b), axis=2))
    return 2.0 * np.arctan2(diff, summ)


def angularity_deg(lat_deg, lon_deg, elev_ft):
    return np.degrees(pairwise_vector_angle(station_vectors(lat_deg, lon_deg, elev_ft)))


def distance_and_angularity(lat_deg, lon_deg, elev_ft):
    """(distance_km, angle_deg), both [N, N] float64, like DataLoader.getDistanceAndAngularity."""
    return haversine_km(lat_deg, lon_deg), angularity_deg(lat_deg, lon_deg, elev_ft)


def metres_to_feet(elev_m):
    """Synthetic elevations are drawn in metres; the reference formula expects feet."""
    return np.asarray(elev_m, dtype=np.float64) / FEET_TO_METRES
